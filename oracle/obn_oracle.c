/*
 * obn_oracle.c — CPU restatement of 0xBitNet's ternary BitLinear path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never part of
 * it. Build with -ffp-contract=off so every float operation rounds exactly
 * once, as the shader source writes it. Citations are relative to the
 * reference project root (m96-chan/0xBitNet).
 */
#include "obn_oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- mulberry32 (packages/core/src/shaders/__tests__/helpers/tensor-utils.ts:9-17)
 * JS keeps `s` as an int32 and uses >>> / Math.imul; all of that is plain
 * modulo-2^32 arithmetic on the bit pattern. */
void orc_mulberry32_seed(orc_rng* r, uint32_t seed) { r->s = seed; }

double orc_mulberry32_next(orc_rng* r) {
  r->s = r->s + 0x6d2b79f5u;
  uint32_t s = r->s;
  uint32_t t = (s ^ (s >> 15)) * (1u | s);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

/* tensor-utils.ts:20-27: rng()*2-1 in double, stored into a Float32Array. */
void orc_randf32(float* out, size_t n, uint32_t seed) {
  orc_rng r; orc_mulberry32_seed(&r, seed);
  for (size_t i = 0; i < n; ++i) out[i] = (float)(orc_mulberry32_next(&r) * 2.0 - 1.0);
}

/* tensor-utils.ts:30-38: thresholds 0.333 / 0.666. */
void orc_rand_ternary(int8_t* out, size_t n, uint32_t seed) {
  orc_rng r; orc_mulberry32_seed(&r, seed);
  for (size_t i = 0; i < n; ++i) {
    double v = orc_mulberry32_next(&r);
    out[i] = (int8_t)(v < 0.333 ? -1 : (v < 0.666 ? 0 : 1));
  }
}

/* tensor-utils.ts:41-48: floor(rng()*255) - 127. */
void orc_rand_int8(int32_t* out, size_t n, uint32_t seed) {
  orc_rng r; orc_mulberry32_seed(&r, seed);
  for (size_t i = 0; i < n; ++i) out[i] = (int32_t)floor(orc_mulberry32_next(&r) * 255.0) - 127;
}

/* ---- I2_S (packages/core/src/shaders/__tests__/helpers/i2s-pack.ts) ---- */
/* i2s-pack.ts:30-58: value v -> code v+1; byte gp of a 128-element block
 * holds elements gp, 32+gp, 64+gp, 96+gp in bits [7:6],[5:4],[3:2],[1:0]. */
size_t orc_i2s_pack_row(const int8_t* values, int K, uint8_t* out) {
  int nblk = (K + 127) / 128;
  for (int b = 0; b < nblk; ++b) {
    for (int gp = 0; gp < 32; ++gp) {
      uint8_t byte = 0;
      for (int g = 0; g < 4; ++g) {
        int k = b * 128 + g * 32 + gp;
        int v = k < K ? values[k] : 0;            /* padding is value 0 (code 1) */
        byte |= (uint8_t)((v + 1) << (6 - 2 * g));
      }
      out[b * 32 + gp] = byte;
    }
  }
  return (size_t)nblk * 32;
}

/* i2s-pack.ts:69-84: u32 = block*8 + gp/4, shift = (gp%4)*8 + 6 - 2*group,
 * read little-endian. Byte (gp%4) of that u32 is byte gp of the block. */
void orc_i2s_unpack_row(const uint8_t* packed, int K, int8_t* out) {
  for (int k = 0; k < K; ++k) {
    int block = k / 128, pos = k % 128, group = pos / 32, gp = pos % 32;
    int u32_idx = block * 8 + gp / 4;
    const uint8_t* p = packed + 4 * u32_idx;
    uint32_t w = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                 ((uint32_t)p[3] << 24);
    int shift = (gp % 4) * 8 + (6 - 2 * group);
    out[k] = (int8_t)((int)((w >> shift) & 3u) - 1);
  }
}

/* i2s-pack.ts:91-103, for K % 128 == 0 (rows of exactly K/4 bytes). */
void orc_i2s_pack_matrix(const int8_t* values, int M, int K, uint8_t* out) {
  for (int m = 0; m < M; ++m)
    orc_i2s_pack_row(values + (size_t)m * K, K, out + (size_t)m * (K / 4));
}

/* ---- RMSNorm (packages/core/src/shaders/rmsnorm.wgsl:40-62) ------------- */
static float rms_factor(const float* xr, int D, float eps) {
  float part[ORC_LANES];
  for (int tid = 0; tid < ORC_LANES; ++tid) {       /* :41-45 strided partials */
    float s = 0.0f;
    for (int col = tid; col < D; col += ORC_LANES) {
      float v = xr[col];
      float sq = v * v;
      s = s + sq;
    }
    part[tid] = s;
  }
  for (int stride = ORC_LANES / 2; stride > 0; stride >>= 1)   /* :50-55 tree */
    for (int tid = 0; tid < stride; ++tid) part[tid] = part[tid] + part[tid + stride];
  float mean = part[0] / (float)D;                  /* :57 */
  float v = mean + eps;
  return 1.0f / sqrtf(v);                           /* inverseSqrt as 1/sqrt, IEEE */
}

void orc_rmsnorm(const float* x, const float* w, int N, int D, float eps, float* y) {
  for (int n = 0; n < N; ++n) {
    const float* xr = x + (size_t)n * D;
    float rms = rms_factor(xr, D, eps);
    for (int col = 0; col < D; ++col) {             /* :60-62 (x*rms)*w */
      float t = xr[col] * rms;
      y[(size_t)n * D + col] = t * w[col];
    }
  }
}

/* ---- Quantize (packages/core/src/shaders/quantize.wgsl:41-73) ----------- */
static void quantize_row(const float* xr, int D, int8_t* qr, float* scale_out) {
  float part[ORC_LANES];
  for (int tid = 0; tid < ORC_LANES; ++tid) {       /* :41-44 */
    float m = 0.0f;
    for (int col = tid; col < D; col += ORC_LANES) m = fmaxf(m, fabsf(xr[col]));
    part[tid] = m;
  }
  for (int stride = ORC_LANES / 2; stride > 0; stride >>= 1)   /* :49-54 */
    for (int tid = 0; tid < stride; ++tid) part[tid] = fmaxf(part[tid], part[tid + stride]);
  float absmax = part[0];
  *scale_out = absmax == 0.0f ? 1.0f : absmax / 127.0f;        /* :59 */
  float inv = absmax == 0.0f ? 0.0f : 127.0f / absmax;         /* :68 */
  for (int col = 0; col < D; ++col) {               /* :69-73 */
    float t = xr[col] * inv;
    float r = rintf(t);                             /* WGSL round(): ties to even */
    int qi = (int)r;
    if (qi < -127) qi = -127;
    if (qi > 127) qi = 127;
    qr[col] = (int8_t)qi;
  }
}

void orc_quantize(const float* x, int N, int D, int8_t* q, float* scales) {
  for (int n = 0; n < N; ++n)
    quantize_row(x + (size_t)n * D, D, q + (size_t)n * D, &scales[n]);
}

/* ---- Ternary integer core (ternary_gemv.wgsl:55-78, ternary_gemm.wgsl:61-119)
 * For each packed u32 col: block = col/8, base_gp = (col%8)*4; byte bi holds
 * elements block*128 + base_gp + bi + {0,32,64,96} in bits [7:6]..[1:0]. */
static int32_t row_dot(const uint8_t* wr, const int8_t* q, int K) {
  int32_t acc = 0;
  int kp = K / 16;                                  /* K_packed u32 per row */
  for (int col = 0; col < kp; ++col) {
    const uint8_t* p = wr + 4 * col;
    int block = col / 8, base_gp = (col % 8) * 4;
    for (int bi = 0; bi < 4; ++bi) {
      uint32_t bv = p[bi];
      int base = block * 128 + base_gp + bi;
      int w0 = (int)((bv >> 6) & 3u) - 1, w1 = (int)((bv >> 4) & 3u) - 1;
      int w2 = (int)((bv >> 2) & 3u) - 1, w3 = (int)(bv & 3u) - 1;
      acc += w0 * q[base] + w1 * q[base + 32] + w2 * q[base + 64] + w3 * q[base + 96];
    }
  }
  return acc;
}

void orc_ternary_acc(const uint8_t* w_i2s, const int8_t* q, int M, int N, int K,
                     int32_t* acc) {
  size_t rb = (size_t)K / 4;
  for (int n = 0; n < N; ++n)
    for (int m = 0; m < M; ++m)
      acc[(size_t)n * M + m] = row_dot(w_i2s + (size_t)m * rb, q + (size_t)n * K, K);
}

/* The same int32 accumulators, faster for large test shapes: each weight row is
 * decoded once (the row_dot decode above: block = col/8, element base_gp + bi +
 * 32 g of the block in bits 7-2g:6-2g of byte bi) and dotted with every token;
 * rows are split over OpenMP threads. Integer sums do not depend on their order,
 * so the result equals orc_ternary_acc exactly. */
void orc_ternary_acc_omp(const uint8_t* w_i2s, const int8_t* q, int M, int N, int K,
                         int32_t* acc, int threads) {
#ifdef _OPENMP
  int nt = threads > 0 ? threads : omp_get_max_threads();
#else
  int nt = 1; (void)threads;
#endif
  size_t rb = (size_t)K / 4;
#pragma omp parallel num_threads(nt)
  {
    int8_t* w = (int8_t*)malloc((size_t)K);
#pragma omp for schedule(static)
    for (int m = 0; m < M; ++m) {
      const uint8_t* wr = w_i2s + (size_t)m * rb;
      for (int col = 0; col < K / 16; ++col) {
        const uint8_t* p = wr + 4 * col;
        int block = col / 8, base_gp = (col % 8) * 4;
        for (int bi = 0; bi < 4; ++bi) {
          uint32_t bv = p[bi];
          int base = block * 128 + base_gp + bi;
          w[base] = (int8_t)((int)((bv >> 6) & 3u) - 1);
          w[base + 32] = (int8_t)((int)((bv >> 4) & 3u) - 1);
          w[base + 64] = (int8_t)((int)((bv >> 2) & 3u) - 1);
          w[base + 96] = (int8_t)((int)(bv & 3u) - 1);
        }
      }
      for (int n = 0; n < N; ++n) {
        const int8_t* qr = q + (size_t)n * K;
        int32_t a = 0;
        for (int k = 0; k < K; ++k) a += (int32_t)w[k] * (int32_t)qr[k];
        acc[(size_t)n * M + m] = a;
      }
    }
    free(w);
  }
}

/* ternary_gemv.wgsl:93-95: sum * scales[row] * input_scale, left to right. */
void orc_ternary_gemv(const uint8_t* w_i2s, const int8_t* q, const float* s_w,
                      float s_x, int M, int K, float* out) {
  size_t rb = (size_t)K / 4;
  for (int m = 0; m < M; ++m) {
    float sum = (float)row_dot(w_i2s + (size_t)m * rb, q, K);
    float t = sum * s_w[m];
    out[m] = t * s_x;
  }
}

/* ternary_gemm.wgsl:128-133: scale = w_scale * input_scales[n]; f32(acc)*scale. */
void orc_ternary_gemm(const uint8_t* w_i2s, const int8_t* q, const float* s_w,
                      const float* s_x, int M, int N, int K, float* out) {
  size_t rb = (size_t)K / 4;
  for (int n = 0; n < N; ++n)
    for (int m = 0; m < M; ++m) {
      float scale = s_w[m] * s_x[n];
      float a = (float)row_dot(w_i2s + (size_t)m * rb, q + (size_t)n * K, K);
      out[(size_t)n * M + m] = a * scale;
    }
}

/* ---- BitLinear::forward (packages/rust/crates/oxbitnet/src/nn/bitlinear.rs:52-97) */
void orc_bitlinear(const float* x, int n, const float* norm_w, float eps,
                   const uint8_t* w_i2s, const float* s_w, int M, int K,
                   float* out, int8_t* q_out, float* s_out) {
  const float* src = x;
  float* normed = NULL;
  if (norm_w) {                                     /* :61-71 */
    normed = (float*)malloc(sizeof(float) * (size_t)n * K);
    orc_rmsnorm(x, norm_w, n, K, eps, normed);
    src = normed;
  }
  int8_t* q = q_out ? q_out : (int8_t*)malloc((size_t)n * K);
  float* sc = s_out ? s_out : (float*)malloc(sizeof(float) * (size_t)n);
  orc_quantize(src, n, K, q, sc);                   /* :73-82 */
  if (n == 1) orc_ternary_gemv(w_i2s, q, s_w, sc[0], M, K, out);   /* :90-91 */
  else        orc_ternary_gemm(w_i2s, q, s_w, sc, M, n, K, out);   /* :92-93 */
  if (!q_out) free(q);
  if (!s_out) free(sc);
  free(normed);
}

/* ---- Gated FFN activation (ffn.rs:70-79) ---------------------------------- */
/* activation.wgsl:30-33 (ReLU^2: max(0, x), squared) on gate, then
 * elementwise.wgsl:31-32 (multiply) by up: y = (r * r) * u. */
void orc_relu2_mul(const float* gate, const float* up, size_t n, float* y) {
  for (size_t i = 0; i < n; ++i) {
    float r = fmaxf(0.0f, gate[i]);
    float t = r * r;
    y[i] = t * up[i];
  }
}

/* ---- RoPE (packages/core/src/shaders/rope.wgsl:27-56) --------------------- */
/* x [N, heads, head_dim] in place: pair i of (token t, head h) at position
 * pos_offset + t rotates by theta = pos * base^(-2i/D) (:43-45). */
void orc_rope(float* x, int N, int heads, int head_dim, int pos_offset, float theta_base) {
  const int half = head_dim / 2;
  for (int t = 0; t < N; ++t)
    for (int h = 0; h < heads; ++h)
      for (int i = 0; i < half; ++i) {
        float pos = (float)(t + pos_offset);
        float freq_exp = -2.0f * (float)i / (float)head_dim;
        float theta = pos * powf(theta_base, freq_exp);
        float c = cosf(theta), sn = sinf(theta);
        float* p = x + ((size_t)t * heads + h) * head_dim + 2 * i;
        float x0 = p[0], x1 = p[1];
        float a = x0 * c, b = x1 * sn, e = x0 * sn, f = x1 * c;
        p[0] = a - b;                                /* :54-55 */
        p[1] = e + f;
      }
}

/* ---- Attention (attention.wgsl + softmax.wgsl, attention.rs:85-124) ------- */
/* One sequence: q [N, H, d]; K, V [S, Hkv, d] (S includes the N new tokens);
 * out [N, H, d]. scores = (sequential dot) * scale with the causal mask
 * k > q + (S - N) -> -FLT_MAX (attention.wgsl:44-56); softmax.wgsl's three
 * passes with 256-lane partials and halving trees; out = sequential sum over
 * s of weight * V (attention.wgsl:87-95). */
void orc_attention(const float* q, const float* K, const float* V, int N, int S, int H, int Hkv,
                   int d, float scale, float* out) {
  float* sc = (float*)malloc(sizeof(float) * (size_t)S);
  float part[ORC_LANES];
  const int group = H / Hkv;
  for (int h = 0; h < H; ++h) {
    const int kvh = h / group;
    for (int t = 0; t < N; ++t) {
      const float* qr = q + ((size_t)t * H + h) * d;
      for (int s = 0; s < S; ++s) {
        const float* kr = K + ((size_t)s * Hkv + kvh) * d;
        float dot = 0.0f;
        for (int i = 0; i < d; ++i) { float pr = qr[i] * kr[i]; dot = dot + pr; }
        sc[s] = (s > t + (S - N)) ? -3.402823e+38f : dot * scale;
      }
      for (int tid = 0; tid < ORC_LANES; ++tid) {   /* softmax pass 1: max */
        float m = -3.402823e+38f;
        for (int c = tid; c < S; c += ORC_LANES) m = fmaxf(m, sc[c]);
        part[tid] = m;
      }
      for (int st = ORC_LANES / 2; st > 0; st >>= 1)
        for (int tid = 0; tid < st; ++tid) part[tid] = fmaxf(part[tid], part[tid + st]);
      const float mx = part[0];
      for (int tid = 0; tid < ORC_LANES; ++tid) {   /* pass 2: sum of exp */
        float acc = 0.0f;
        for (int c = tid; c < S; c += ORC_LANES) acc = acc + expf(sc[c] - mx);
        part[tid] = acc;
      }
      for (int st = ORC_LANES / 2; st > 0; st >>= 1)
        for (int tid = 0; tid < st; ++tid) part[tid] = part[tid] + part[tid + st];
      const float inv = 1.0f / part[0];
      for (int s = 0; s < S; ++s) sc[s] = expf(sc[s] - mx) * inv;   /* pass 3 */
      float* orow = out + ((size_t)t * H + h) * d;
      for (int i = 0; i < d; ++i) {
        float sum = 0.0f;
        for (int s = 0; s < S; ++s) { float pr = sc[s] * V[((size_t)s * Hkv + kvh) * d + i]; sum = sum + pr; }
        orow[i] = sum;
      }
    }
  }
  free(sc);
}

/* ---- LM head (packages/core/src/shaders/f32_matmul.wgsl:27-74) ---------- */
/* IEEE binary16 -> binary32, exact (unpack2x16float). */
float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  if (e == 0x1Fu) {
    bits = sign | 0x7F800000u | (m << 13);            /* inf / nan */
  } else if (e != 0) {
    bits = sign | ((e + 112u) << 23) | (m << 13);     /* normal: rebias 15 -> 127 */
  } else if (m == 0) {
    bits = sign;                                      /* signed zero */
  } else {                                            /* subnormal: normalise */
    int shift = 0;
    while (!(m & 0x400u)) { m <<= 1; ++shift; }
    bits = sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* logits[n, v] = sum_d hidden[n, d] * f32(embed[v, d]), the shader's order: lane
 * tid of 256 accumulates the d-pairs dh = tid, tid + 256, ... (two products per
 * pair, :51-57), then the halving tree (:63-68). embed [V, D] binary16. */
void orc_lm_head_f16(const float* hidden, const uint16_t* embed, int N, int V, int D,
                     float* out) {
  const int dh_n = D / 2;
  for (int n = 0; n < N; ++n) {
    const float* h = hidden + (size_t)n * D;
    /* logits are independent: split over threads, each with its own lanes */
#pragma omp parallel for schedule(static)
    for (int v = 0; v < V; ++v) {
      float part[ORC_LANES];
      const uint16_t* e = embed + (size_t)v * D;
      for (int tid = 0; tid < ORC_LANES; ++tid) {
        float acc = 0.0f;
        for (int dh = tid; dh < dh_n; dh += ORC_LANES) {
          const int d = dh * 2;
          float t0 = h[d] * orc_half_to_float(e[d]);
          acc = acc + t0;
          float t1 = h[d + 1] * orc_half_to_float(e[d + 1]);
          acc = acc + t1;
        }
        part[tid] = acc;
      }
      for (int stride = ORC_LANES / 2; stride > 0; stride >>= 1)
        for (int tid = 0; tid < stride; ++tid) part[tid] = part[tid] + part[tid + stride];
      out[(size_t)n * V + v] = part[0];
    }
  }
}

/* The TS test helper refF32Matmul (helpers/reference.ts:342-360): one
 * sequential sum over d with an f32 embedding. */
void orc_f32_matmul_seq(const float* hidden, const float* embed, int N, int V, int D, float* out) {
  for (int n = 0; n < N; ++n)
    for (int v = 0; v < V; ++v) {
      float sum = 0.0f;
      for (int d = 0; d < D; ++d) {
        float t = hidden[(size_t)n * D + d] * embed[(size_t)v * D + d];
        sum = sum + t;
      }
      out[(size_t)n * V + v] = sum;
    }
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Row-parallel version of orc_bitlinear for the timed CPU baseline: the same
 * per-element arithmetic, split over tokens (norm/quantize) and over output
 * rows (GEMV/GEMM), so results are identical to orc_bitlinear. */
void orc_bitlinear_omp(const float* x, int n, const float* norm_w, float eps,
                       const uint8_t* w_i2s, const float* s_w, int M, int K,
                       float* out, int threads) {
#ifdef _OPENMP
  int nt = threads > 0 ? threads : omp_get_max_threads();
#else
  int nt = 1; (void)threads;
#endif
  float* normed = (float*)malloc(sizeof(float) * (size_t)n * K);
  int8_t* q = (int8_t*)malloc((size_t)n * K);
  float* sc = (float*)malloc(sizeof(float) * (size_t)n);
  size_t rb = (size_t)K / 4;
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int t = 0; t < n; ++t) {
    const float* xr = x + (size_t)t * K;
    if (norm_w) { orc_rmsnorm(xr, norm_w, 1, K, eps, normed + (size_t)t * K); xr = normed + (size_t)t * K; }
    quantize_row(xr, K, q + (size_t)t * K, &sc[t]);
  }
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int m = 0; m < M; ++m) {
    const uint8_t* wr = w_i2s + (size_t)m * rb;
    for (int t = 0; t < n; ++t) {
      float a = (float)row_dot(wr, q + (size_t)t * K, K);
      if (n == 1) { float u = a * s_w[m]; out[m] = u * sc[0]; }
      else { float scale = s_w[m] * sc[t]; out[(size_t)t * M + m] = a * scale; }
    }
  }
  free(normed); free(q); free(sc);
}
