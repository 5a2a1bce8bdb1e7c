"""Pins the CPU oracle against the reference's own known-answer tests.

Every case restates one vitest case from the reference
(packages/core/src/shaders/__tests__/*.test.ts, cited per test) with the same
seeded inputs (mulberry32 restated in oracle/obn_oracle.c) and the same
assertions and tolerances (expectClose: rtol 1e-5, atol 1e-6 unless the
reference passes others). CPU only.
"""
import math

import numpy as np
import pytest

import oracle as orc


def expect_close(actual, expected, rtol=1e-5, atol=1e-6):
    """tensor-utils.ts:51-68."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    assert a.shape == e.shape
    tol = atol + rtol * np.abs(e)
    bad = np.abs(a - e) > tol
    assert not bad.any(), f"mismatch at {np.flatnonzero(bad)[:5]}: {a[bad][:5]} vs {e[bad][:5]}"


def pack_matrix_rows(rows, K):
    return np.stack([orc.i2s_pack_row(np.asarray(r, np.int8), K) for r in rows])


def naive_gemv(packed, q, s_w, s_x, M, K):
    """refTernaryGemvNaive (reference.ts:80-103): unpack, dot in double."""
    out = np.empty(M, np.float32)
    for m in range(M):
        w = orc.i2s_unpack_row(packed[m], K).astype(np.int64)
        acc = float(np.dot(w, np.asarray(q, np.int64)))
        out[m] = np.float32(acc * float(s_w[m]) * float(s_x))
    return out


# ---------------------------------------------------------------- generators
def test_mulberry32_is_deterministic_and_in_range():
    a = orc.randf32(1000, 42)
    b = orc.randf32(1000, 42)
    assert np.array_equal(a, b)
    assert a.min() >= -1.0 and a.max() < 1.0
    t = orc.rand_ternary(3000, 7)
    assert set(np.unique(t).tolist()) == {-1, 0, 1}
    i = orc.rand_int8(3000, 7)
    assert i.min() >= -127 and i.max() <= 127


def test_mulberry32_first_value_seed_42():
    # Hand evaluation of tensor-utils.ts:9-17 for seed 42:
    # s = 42 + 0x6d2b79f5; t = imul(s ^ s>>>15, 1|s); t = (t + imul(t ^ t>>>7, 61|t)) ^ t;
    # (t ^ t>>>14) >>> 0, all modulo 2^32.
    s = (42 + 0x6D2B79F5) & 0xFFFFFFFF
    t = ((s ^ (s >> 15)) * (1 | s)) & 0xFFFFFFFF
    t = ((t + (((t ^ (t >> 7)) * (61 | t)) & 0xFFFFFFFF)) & 0xFFFFFFFF) ^ t
    want = ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0
    got = orc.randf32(1, 42)[0]
    assert got == np.float32(want * 2 - 1)


# ---------------------------------------------------------------- I2_S
# i2s-pack.test.ts
def test_i2s_round_trip_known_pattern():  # :6-19
    v = np.zeros(128, np.int8)
    v[0], v[1], v[32], v[64], v[96] = -1, 1, 1, -1, 1
    assert np.array_equal(orc.i2s_unpack_row(orc.i2s_pack_row(v, 128), 128), v)


@pytest.mark.parametrize("K,seed", [(128, 1), (256, 2), (384, 3)])
def test_i2s_round_trip_random(K, seed):  # :21-40
    v = orc.rand_ternary(K, seed)
    assert np.array_equal(orc.i2s_unpack_row(orc.i2s_pack_row(v, K), K), v)


def test_i2s_round_trip_non_aligned_200():  # :42-48
    v = orc.rand_ternary(200, 4)
    packed = orc.i2s_pack_row(v, 200)
    assert packed.size == 64  # padded to 256 elements
    assert np.array_equal(orc.i2s_unpack_row(packed, 200), v)


def test_i2s_round_trip_matrix():  # :50-62
    M, K = 4, 256
    rows = np.stack([orc.rand_ternary(K, 10 + m) for m in range(M)])
    packed = orc.i2s_pack_matrix(rows)
    assert np.array_equal(orc.i2s_unpack_matrix(packed, K), rows)


@pytest.mark.parametrize("val,word", [(-1, 0x00000000), (1, 0xAAAAAAAA), (0, 0x55555555)])
def test_i2s_known_byte_layout(val, word):  # :64-85
    packed = orc.i2s_pack_row(np.full(128, val, np.int8), 128)
    assert int(packed[:4].view("<u4")[0]) == word


# ---------------------------------------------------------------- quantize
# quantize.test.ts
def test_quantize_simple_known_values():  # :6-19
    q, s = orc.quantize(np.array([[1.0, -1.0, 0.5, 0.0]], np.float32))
    assert abs(s[0] - 1 / 127) < 1e-6
    assert q[0].tolist() == [127, -127, 64, 0]


def test_quantize_scale_formula():  # :21-29
    _, s = orc.quantize(np.array([[3.0, -5.0, 2.0, 1.0]], np.float32))
    expect_close([s[0]], [5 / 127], 1e-6)


def test_quantize_clamped():  # :31-41
    q, _ = orc.quantize(np.array([[10, -10, 5]], np.float32))
    assert q.min() >= -127 and q.max() <= 127


def test_quantize_zero_row():  # :43-53
    q, s = orc.quantize(np.zeros((1, 4), np.float32))
    assert s[0] == 1.0 and not q.any()


def test_quantize_per_token_scales():  # :55-66
    _, s = orc.quantize(np.array([[1, 2, 3], [10, 5, 1]], np.float32))
    expect_close([s[0]], [3 / 127], 1e-6)
    expect_close([s[1]], [10 / 127], 1e-6)


def test_quantize_dequant_error():  # :68-83
    N, D = 4, 128
    x = orc.randf32(N * D, 42).reshape(N, D)
    q, s = orc.quantize(x)
    err = np.abs(x - q.astype(np.float32) * s[:, None])
    assert (err < s[:, None] * 1.5).all()


def test_quantize_rounds_ties_to_even():
    # WGSL round() (quantize.wgsl:71) is ties-to-even. The TS helper's
    # Math.round (reference.ts:70) rounds ties up and would give -63 / 3 here;
    # the shader, which is what runs, is the contract.
    x = np.array([[127.0, -63.5, 2.5, 0.5, -0.5, 1.5]], np.float32)
    q, s = orc.quantize(x)
    assert s[0] == np.float32(127.0) / np.float32(127.0)
    assert q[0].tolist() == [127, -64, 2, 0, 0, 2]


# ---------------------------------------------------------------- RMSNorm
# rmsnorm.test.ts
def test_rmsnorm_unit_weight():  # :6-18
    x = np.array([[1, 2, 3, 4]], np.float32)
    y = orc.rmsnorm(x, np.ones(4, np.float32), 1e-5)
    rms = math.sqrt(30 / 4 + 1e-5)
    expect_close(y, [1 / rms, 2 / rms, 3 / rms, 4 / rms], 1e-5)


def test_rmsnorm_weight_scaling():  # :20-31
    x = np.array([[1, 2, 3, 4]], np.float32)
    y2 = orc.rmsnorm(x, np.full(4, 2, np.float32))
    y1 = orc.rmsnorm(x, np.ones(4, np.float32))
    expect_close(y2, y1 * 2, 1e-5)


def test_rmsnorm_multiple_rows():  # :33-47
    x = np.array([[1, 2, 3, 4], [-1, -2, -3, -4]], np.float32)
    y = orc.rmsnorm(x, np.ones(4, np.float32))
    expect_close(y[1], -y[0], 1e-5)


def test_rmsnorm_zero_input():  # :49-59
    y = orc.rmsnorm(np.zeros((1, 4), np.float32), np.ones(4, np.float32))
    expect_close(y, np.zeros(4))


def test_rmsnorm_random_shape():  # :61-68
    x = orc.randf32(8 * 512, 42).reshape(8, 512)
    w = orc.randf32(512, 43)
    assert orc.rmsnorm(x, w).shape == (8, 512)


def test_rmsnorm_reduction_order_is_the_shaders():
    # The restatement reduces 256 strided lane partials then a halving tree
    # (rmsnorm.wgsl:41-55). Check it against an explicit numpy float32 replay.
    D = 2560
    x = orc.randf32(D, 5)
    w = np.ones(D, np.float32)
    part = np.zeros(256, np.float32)
    for tid in range(256):
        s = np.float32(0)
        for col in range(tid, D, 256):
            s = np.float32(s + np.float32(x[col] * x[col]))
        part[tid] = s
    stride = 128
    while stride:
        part[:stride] = (part[:stride] + part[stride:2 * stride]).astype(np.float32)
        stride //= 2
    rms = np.float32(1) / np.sqrt(np.float32(part[0] / np.float32(D)) + np.float32(1e-5))
    want = (x * rms).astype(np.float32) * w
    assert np.array_equal(orc.rmsnorm(x[None], w)[0], want)


# ---------------------------------------------------------------- GEMV
# ternary-gemv.test.ts
def _gemv_setup(seed=42, M=8, K=256):  # :13-26
    rows = [orc.rand_ternary(K, seed + m) for m in range(M)]
    packed = pack_matrix_rows(rows, K)
    q = orc.rand_int8(K, seed + 100).astype(np.int8)
    s_w = np.array([0.01 + 0.001 * m for m in range(M)], np.float32)
    return rows, packed, q, s_w, np.float32(0.05)


def test_gemv_naive_vs_shader_logic():  # :28-33
    _, packed, q, s_w, s_x = _gemv_setup()
    expect_close(orc.ternary_gemv(packed, q, s_w, s_x, 8, 256),
                 naive_gemv(packed, q, s_w, s_x, 8, 256), 1e-5)


def test_gemv_known_k128():  # :35-53
    packed = pack_matrix_rows([np.ones(128), -np.ones(128)], 128)
    out = orc.ternary_gemv(packed, np.ones(128, np.int8), np.ones(2, np.float32), 1.0, 2, 128)
    assert out.tolist() == [128.0, -128.0]


def test_gemv_zero_weights():  # :55-64
    packed = pack_matrix_rows([np.zeros(256)] * 8, 256)
    q = orc.rand_int8(256, 1).astype(np.int8)
    assert not orc.ternary_gemv(packed, q, np.ones(8, np.float32), 1.0, 8, 256).any()


def test_gemv_scale_applied():  # :66-77
    _, packed, q, _, s_x = _gemv_setup()
    a = orc.ternary_gemv(packed, q, np.ones(8, np.float32), s_x, 8, 256)
    b = orc.ternary_gemv(packed, q, np.full(8, 2, np.float32), s_x, 8, 256)
    expect_close(b, a * 2, 1e-5)


def test_gemv_k384():  # :79-94
    rows = [orc.rand_ternary(384, 50 + m) for m in range(4)]
    packed = pack_matrix_rows(rows, 384)
    q = orc.rand_int8(384, 200).astype(np.int8)
    s_w = np.full(4, 0.01, np.float32)
    expect_close(orc.ternary_gemv(packed, q, s_w, 0.03, 4, 384),
                 naive_gemv(packed, q, s_w, 0.03, 4, 384), 1e-5)


# ---------------------------------------------------------------- GEMM
# ternary-gemm.test.ts
def test_gemm_n1_matches_gemv():  # :10-35
    rows = [orc.rand_ternary(256, 10 + m) for m in range(8)]
    packed = pack_matrix_rows(rows, 256)
    q = orc.rand_int8(256, 100).astype(np.int8)
    s_w = np.array([0.01 + 0.001 * m for m in range(8)], np.float32)
    g = orc.ternary_gemm(packed, q[None], s_w, np.array([0.05], np.float32), 8, 256)
    expect_close(g[0], orc.ternary_gemv(packed, q, s_w, 0.05, 8, 256), 1e-5)


def test_gemm_output_layout():  # :37-72
    M, K, N = 4, 128, 3
    packed = pack_matrix_rows([orc.rand_ternary(K, 20 + m) for m in range(M)], K)
    q = orc.rand_int8(N * K, 200).astype(np.int8).reshape(N, K)
    s_w = np.full(M, 0.01, np.float32)
    s_x = np.array([0.01 + 0.005 * n for n in range(N)], np.float32)
    out = orc.ternary_gemm(packed, q, s_w, s_x, M, K)
    assert out.size == N * M
    for n in range(N):
        expect_close(out[n], naive_gemv(packed, q[n], s_w, s_x[n], M, K), 1e-5)


def test_gemm_per_token_scales():  # :74-96
    M, K, N = 4, 128, 2
    packed = pack_matrix_rows([orc.rand_ternary(K, 30 + m) for m in range(M)], K)
    q = orc.rand_int8(N * K, 300).astype(np.int8).reshape(N, K)
    ones = np.ones(M, np.float32)
    a = orc.ternary_gemm(packed, q, ones, np.array([1, 1], np.float32), M, K)
    b = orc.ternary_gemm(packed, q, ones, np.array([2, 3], np.float32), M, K)
    expect_close(b[0], a[0] * 2, 1e-5)
    expect_close(b[1], a[1] * 3, 1e-5)


def test_gemm_known_pm128():  # :98-121
    packed = pack_matrix_rows([np.ones(128), -np.ones(128)], 128)
    out = orc.ternary_gemm(packed, np.ones((2, 128), np.int8), np.ones(2, np.float32),
                           np.ones(2, np.float32), 2, 128)
    assert out.tolist() == [[128.0, -128.0], [128.0, -128.0]]


def test_gemm_k384_multiblock():  # :123-152
    M, K, N = 4, 384, 2
    packed = pack_matrix_rows([orc.rand_ternary(K, 40 + m) for m in range(M)], K)
    q = orc.rand_int8(N * K, 400).astype(np.int8).reshape(N, K)
    s_w = np.full(M, 0.01, np.float32)
    s_x = np.full(N, 0.02, np.float32)
    out = orc.ternary_gemm(packed, q, s_w, s_x, M, K)
    for n in range(N):
        expect_close(out[n], naive_gemv(packed, q[n], s_w, s_x[n], M, K), 1e-5)


# ---------------------------------------------------------------- BitLinear e2e
# bitlinear-e2e.test.ts
def test_e2e_identity_like():  # :81-109
    K, M = 128, 64
    x = orc.randf32(K, 1)
    rows = np.zeros((M, K), np.int8)
    rows[np.arange(M), np.arange(M)] = 1
    out, _, _ = orc.bitlinear(x, orc.i2s_pack_matrix(rows), np.ones(M, np.float32), M, K)
    assert out.shape == (1, M)
    assert (np.abs(out) > 1e-10).sum() > M / 2


def test_e2e_gemv_matches_gemm_n1():  # :111-139
    K, M = 256, 128
    x = orc.randf32(K, 10)
    packed = orc.i2s_pack_matrix(np.stack([orc.rand_ternary(K, 100 + i) for i in range(M)]))
    s_w = np.ones(M, np.float32)
    gemv, _, _ = orc.bitlinear(x, packed, s_w, M, K)
    q, s = orc.quantize(x[None])
    gemm = orc.ternary_gemm(packed, q, s_w, s, M, K)
    expect_close(gemv, gemm, 1e-5, 1e-6)


def test_e2e_batched():  # :141-163
    K, M, N = 128, 64, 4
    x = orc.randf32(N * K, 20).reshape(N, K)
    packed = orc.i2s_pack_matrix(np.stack([orc.rand_ternary(K, 200 + i) for i in range(M)]))
    out, _, _ = orc.bitlinear(x, packed, np.ones(M, np.float32), M, K)
    assert out.shape == (N, M)
    assert np.abs(out[0] - out[1]).sum() > 0.01


def test_e2e_with_rmsnorm():  # :165-190
    K, M = 128, 64
    x = orc.randf32(K, 30)
    packed = orc.i2s_pack_matrix(np.stack([orc.rand_ternary(K, 300 + i) for i in range(M)]))
    s_w = np.ones(M, np.float32)
    a, _, _ = orc.bitlinear(x, packed, s_w, M, K, norm_w=np.ones(K, np.float32))
    b, _, _ = orc.bitlinear(x, packed, s_w, M, K)
    assert np.abs(a - b).max() > 0.001


def test_e2e_dequant_formula_constant_half():  # :192-217
    K = 256
    out, _, _ = orc.bitlinear(np.full(K, 0.5, np.float32),
                              orc.i2s_pack_matrix(np.ones((1, K), np.int8)),
                              np.ones(1, np.float32), 1, K)
    assert abs(out[0, 0] - 128) < 0.5


def test_e2e_weight_scale_one():  # :219-243
    K, M = 128, 32
    x = orc.randf32(K, 50)
    tern = np.stack([orc.rand_ternary(K, 500 + i) for i in range(M)])
    out, _, _ = orc.bitlinear(x, orc.i2s_pack_matrix(tern), np.ones(M, np.float32), M, K)
    q, s = orc.quantize(x[None])
    expected = float(np.dot(tern[0].astype(np.int64), q[0].astype(np.int64))) * 1.0 * float(s[0])
    assert abs(out[0, 0] - expected) < 0.5e-3


# ---------------------------------------------------------------- OpenMP twin
def test_bitlinear_omp_identical():
    K, M = 512, 96
    packed = orc.i2s_pack_matrix(orc.rand_ternary(M * K, 9).reshape(M, K))
    s_w = np.full(M, 1.25, np.float32)
    g = orc.randf32(K, 3) * 0.1 + 1
    for n in (1, 5):
        x = orc.randf32(n * K, 11 + n).reshape(n, K)
        ref, _, _ = orc.bitlinear(x, packed, s_w, M, K, norm_w=g)
        assert np.array_equal(orc.bitlinear_omp(x, packed, s_w, M, K, norm_w=g, threads=4), ref)


# ---- LM head: f32-matmul.test.ts (refF32Matmul) and the f16 shader order ----
# packages/core/src/shaders/__tests__/f32-matmul.test.ts


def test_f32_matmul_simple_dot_products():  # :6-21
    out = orc.f32_matmul_seq(np.array([1, 2, 3], np.float32),
                             np.array([1, 0, 0, 0, 1, 0], np.float32), 1, 2, 3)
    assert out.tolist() == [1.0, 2.0]


def test_f32_matmul_layout_and_tokens():  # :23-54
    assert orc.f32_matmul_seq(orc.randf32(8, 1), orc.randf32(12, 2), 2, 3, 4).shape == (6,)
    out = orc.f32_matmul_seq(np.array([1, 0, 0, 1, 1, 1], np.float32),
                             np.array([1, 0, 0, 1], np.float32), 3, 2, 2)
    assert out.tolist() == [1, 0, 0, 1, 1, 1]


def test_f32_matmul_zero_hidden():  # :56-68
    out = orc.f32_matmul_seq(np.zeros(4, np.float32), orc.randf32(20, 3), 1, 5, 4)
    assert np.all(out == 0)


def test_f32_matmul_manual_dot():  # :70-89
    h, e = orc.randf32(16, 10), orc.randf32(24, 20)
    out = orc.f32_matmul_seq(h, e, 2, 3, 8)
    want = (h.reshape(2, 8).astype(np.float64) @ e.reshape(3, 8).astype(np.float64).T).ravel()
    np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-6)


def test_lm_head_f16_shader_order_agrees_with_helper():
    # the shader (f16 table, 256-lane partials + tree) against the TS helper
    # (one sequential sum) on a table exactly representable in f16
    N, V, D = 2, 7, 2560
    h = orc.randf32(N * D, 5).reshape(N, D)
    e16 = orc.randf32(V * D, 6).astype(np.float16).reshape(V, D)
    out = orc.lm_head_f16(h, e16)
    seq = orc.f32_matmul_seq(h, e16.astype(np.float32), N, V, D).reshape(N, V)
    e64 = e16.astype(np.float64)
    exact = h.astype(np.float64) @ e64.T
    l1 = np.abs(h.astype(np.float64)) @ np.abs(e64).T
    # both orders stay within f32 summation error of the exact dot product
    # (about 20 roundings for the 256-lane tree, D for the sequential sum)
    assert np.all(np.abs(out - exact) <= 4e-6 * l1)
    assert np.all(np.abs(seq - exact) <= D * 6e-8 * l1)
    # identity rows pick single hidden entries exactly
    eye = np.zeros((3, D), np.float16)
    eye[0, 0] = eye[1, 1] = eye[2, D - 1] = 1
    assert orc.lm_head_f16(h[:1], eye).tolist() == [[h[0, 0], h[0, 1], h[0, D - 1]]]
    assert np.all(orc.lm_head_f16(np.zeros((1, D), np.float32), e16) == 0)


def test_lm_head_f16_with_final_norm():
    D = 256
    x = orc.randf32(D, 7).reshape(1, D)
    g = (1 + 0.1 * orc.randf32(D, 8)).astype(np.float32)
    e16 = orc.randf32(3 * D, 9).astype(np.float16).reshape(3, D)
    assert np.array_equal(orc.lm_head_f16(x, e16, g, 1e-5),
                          orc.lm_head_f16(orc.rmsnorm(x, g, 1e-5), e16))


def test_half_to_float_exact():
    bits = np.arange(0, 65536, 7, dtype=np.uint16)
    finite = bits[np.isfinite(bits.view(np.float16))]
    got = np.array([orc.half_to_float(int(b)) for b in finite], np.float32)
    assert np.array_equal(got, finite.view(np.float16).astype(np.float32))


# ---- gated FFN activation: activation.test.ts / elementwise.test.ts ---------
def test_relu2_mul():
    g = np.array([-2.0, -0.0, 0.0, 0.5, 3.0], np.float32)
    u = np.array([7.0, 1.0, 1.0, 2.0, -1.0], np.float32)
    assert orc.relu2_mul(g, u).tolist() == [0.0, 0.0, 0.0, 0.5, -9.0]


# ---- RoPE / attention: rope.test.ts, softmax.test.ts, attention-*.test.ts ---
def test_rope_position_zero_is_identity():  # rope.test.ts:6-15
    x = orc.randf32(8, 1).reshape(1, 8)
    assert np.allclose(orc.rope(x, 2, 4, 0, 10000.0), x, atol=1e-5)


def test_rope_preserves_pair_norms_and_offset_shifts():  # rope.test.ts:17-51
    x = orc.randf32(16, 2).reshape(1, 16)
    y = orc.rope(x, 2, 8, 5, 10000.0)
    n_in = np.hypot(x[0, 0::2], x[0, 1::2])
    n_out = np.hypot(y[0, 0::2], y[0, 1::2])
    assert np.all(np.abs(n_in - n_out) < 1e-5)
    assert not np.allclose(orc.rope(x[:, :4], 1, 4, 3, 10000.0)[0, 0], x[0, 0], atol=1e-3)


def test_attention_single_key_returns_v():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 4 * 8)).astype(np.float32)
    K = rng.standard_normal((1, 2 * 8)).astype(np.float32)
    V = rng.standard_normal((1, 2 * 8)).astype(np.float32)
    out = orc.attention(q, K, V, 4, 2, 8).reshape(4, 8)
    Vh = V.reshape(2, 8)
    assert np.array_equal(out, np.stack([Vh[h // 2] for h in range(4)]))  # GQA grouping


def test_attention_causal_first_query_sees_first_key():  # attention-scores.test.ts causal
    rng = np.random.default_rng(1)
    q = rng.standard_normal((3, 8)).astype(np.float32)
    K = rng.standard_normal((3, 8)).astype(np.float32)
    V = rng.standard_normal((3, 8)).astype(np.float32)
    out = orc.attention(q, K, V, 1, 1, 8)
    assert np.array_equal(out[0], V[0])


def test_attention_uniform_scores_average_v():  # softmax.test.ts uniform
    V = np.arange(12, dtype=np.float32).reshape(4, 3)
    out = orc.attention(np.zeros((1, 3), np.float32), np.zeros((4, 3), np.float32), V, 1, 1, 3)
    np.testing.assert_allclose(out[0], V.mean(0), rtol=1e-6)


@pytest.mark.parametrize("M,K,N", [(1, 128, 1), (100, 256, 7), (300, 640, 33), (17, 6912, 3)])
def test_openmp_accumulators_equal_the_shader_restatement(M, K, N):
    # orc_ternary_acc_omp (rows decoded once, OpenMP) is the checker of the large
    # GPU parity shapes; it must equal the shader-order orc_ternary_acc exactly.
    rng = np.random.default_rng(M * K + N)
    w = rng.integers(0, 256, (M, K // 4), dtype=np.uint8)
    q = rng.integers(-127, 128, (N, K), dtype=np.int8)
    assert np.array_equal(orc.ternary_acc_omp(w, q, M, K), orc.ternary_acc(w, q, M, K))
