/*
 * obn_oracle.h — CPU restatement of 0xBitNet's ternary BitLinear path.
 *
 * TEST INFRASTRUCTURE ONLY. This header and obn_oracle.c are the checker the
 * parity tests, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm compare the CUDA library against. Nothing in the shipped library
 * (0xbitnet_b200/) includes, links or calls it.
 *
 * Every function restates the arithmetic of one reference WGSL shader or test
 * helper, in the shader's own reduction order, with IEEE single-precision
 * operations and no FMA contraction (the build passes -ffp-contract=off):
 *
 *   orc_rmsnorm          packages/core/src/shaders/rmsnorm.wgsl:40-62
 *   orc_quantize         packages/core/src/shaders/quantize.wgsl:41-73
 *   orc_ternary_gemv     packages/core/src/shaders/ternary_gemv.wgsl:55-96
 *   orc_ternary_gemm     packages/core/src/shaders/ternary_gemm.wgsl:56-135
 *   orc_bitlinear        packages/rust/crates/oxbitnet/src/nn/bitlinear.rs:52-97
 *   orc_i2s_pack_row     packages/core/src/shaders/__tests__/helpers/i2s-pack.ts:30-58
 *   orc_i2s_unpack_row   packages/core/src/shaders/__tests__/helpers/i2s-pack.ts:69-84
 *   orc_mulberry32_*     packages/core/src/shaders/__tests__/helpers/tensor-utils.ts:9-48
 *
 * Parity pin: the reference's own WGSL cannot execute in this environment (no
 * wgpu, no graphics stack, no software adapter), and its TypeScript CPU
 * helpers need node, which is absent. The restatement is pinned against every
 * known-answer test the reference's vitest suite holds for this path
 * (tests/test_oracle_kat.py lists them with their file:line).
 */
#ifndef OBN_ORACLE_H
#define OBN_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number of lanes the reference shaders reduce over (WORKGROUP_SIZE). */
#define ORC_LANES 256

/* ---- seeded generators (tensor-utils.ts:9-48) ------------------------- */
typedef struct { uint32_t s; } orc_rng;
void   orc_mulberry32_seed(orc_rng* r, uint32_t seed);
double orc_mulberry32_next(orc_rng* r);
void   orc_randf32(float* out, size_t n, uint32_t seed);
void   orc_rand_ternary(int8_t* out, size_t n, uint32_t seed);
void   orc_rand_int8(int32_t* out, size_t n, uint32_t seed);

/* ---- I2_S layout (i2s-pack.ts) ---------------------------------------- */
/* Packs K ternary values (padded with 0 to a multiple of 128) into
 * ceil(K/128)*32 bytes. Returns the number of bytes written. */
size_t orc_i2s_pack_row(const int8_t* values, int K, uint8_t* out);
/* Unpacks K values with the shader's block/group/gp formula. */
void   orc_i2s_unpack_row(const uint8_t* packed, int K, int8_t* out);
/* Packs an [M, K] matrix, K % 128 == 0, rows of K/4 bytes. */
void   orc_i2s_pack_matrix(const int8_t* values, int M, int K, uint8_t* out);

/* ---- kernels ------------------------------------------------------------ */
/* rmsnorm.wgsl: y[n,d] = (x[n,d] * rms) * w[d], rms = 1/sqrt(sum/D + eps),
 * sum reduced as 256 strided lane partials then a halving tree. */
void orc_rmsnorm(const float* x, const float* w, int N, int D, float eps, float* y);

/* quantize.wgsl: per-row absmax; scale = absmax==0 ? 1 : absmax/127;
 * q = clamp(round_half_even(x * (absmax==0 ? 0 : 127/absmax)), -127, 127).
 * q is written as int8 (the reference stores the same values as i32). */
void orc_quantize(const float* x, int N, int D, int8_t* q, float* scales);

/* Integer core shared by GEMV and GEMM: acc[n*M + m] = sum_k t[m,k]*q[n,k],
 * t decoded from I2_S rows of K/4 bytes. */
void orc_ternary_acc(const uint8_t* w_i2s, const int8_t* q, int M, int N, int K,
                     int32_t* acc);
/* orc_ternary_acc with each row decoded once and rows split over OpenMP threads
 * (threads <= 0: all); identical results. */
void orc_ternary_acc_omp(const uint8_t* w_i2s, const int8_t* q, int M, int N, int K,
                         int32_t* acc, int threads);

/* ternary_gemv.wgsl: out[m] = (f32(acc[m]) * s_w[m]) * s_x.
 * acc is reduced per row exactly as the shader does (int, order-free). */
void orc_ternary_gemv(const uint8_t* w_i2s, const int8_t* q, const float* s_w,
                      float s_x, int M, int K, float* out);

/* ternary_gemm.wgsl: out[n*M + m] = f32(acc[n,m]) * (s_w[m] * s_x[n]). */
void orc_ternary_gemm(const uint8_t* w_i2s, const int8_t* q, const float* s_w,
                      const float* s_x, int M, int N, int K, float* out);

/* bitlinear.rs:52-97: optional RMSNorm (eps 1e-5 in the reference), quantize,
 * then GEMV when n == 1 and GEMM otherwise. norm_w may be NULL.
 * q_out / s_out (nullable) receive the quantized activations and scales. */
void orc_bitlinear(const float* x, int n, const float* norm_w, float eps,
                   const uint8_t* w_i2s, const float* s_w, int M, int K,
                   float* out, int8_t* q_out, float* s_out);

/* Same as orc_bitlinear with rows split over `threads` OpenMP threads
 * (threads <= 0: all available). Results are identical to orc_bitlinear. */
void orc_bitlinear_omp(const float* x, int n, const float* norm_w, float eps,
                       const uint8_t* w_i2s, const float* s_w, int M, int K,
                       float* out, int threads);

void orc_relu2_mul(const float* gate, const float* up, size_t n, float* y);
void orc_rope(float* x, int N, int heads, int head_dim, int pos_offset, float theta_base);
void orc_attention(const float* q, const float* K, const float* V, int N, int S, int H, int Hkv,
                   int d, float scale, float* out);
float orc_half_to_float(uint16_t h);
void orc_lm_head_f16(const float* hidden, const uint16_t* embed, int N, int V, int D, float* out);
void orc_f32_matmul_seq(const float* hidden, const float* embed, int N, int V, int D, float* out);
int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
