"""Config-2 parity at the sizes the prefill benchmark runs.

The bench times the five BitNet-2B shapes at 512, 2048 and 8192 prefill tokens
(ternary_gemm.wgsl:40-135, dispatched by bitlinear.rs:92-93). These cases run
the persistent tcgen05 GEMM through many tiles per CTA with 20 (K = 2560) or 54
(K = 6912) K blocks per tile, so its stage ring and its double-buffered TMEM
accumulators wrap many times inside one launch. Each case checks, against the
oracle on the same seeded inputs:

* the full int32 accumulator matrix [tokens, rows] (obn_ternary_acc), bit-exact,
  against the oracle's OpenMP accumulators (equal to the shader-order ones,
  tests/test_oracle_kat.py);
* the whole BitLinear forward (fused RMSNorm + int8 quantize + GEMM): the int8
  activations and per-token scales bit-exact, and the f32 outputs against the
  shader's epilogue f32(acc) * (s_w * s_x) (ternary_gemm.wgsl:132-133) applied to
  the oracle accumulators: bit-identical, so within the 1e-5 relative bound.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu

CASES = [("gate", 6912, 2560, 2048), ("down", 2560, 6912, 2048),
         ("gate", 6912, 2560, 8192), ("down", 2560, 6912, 8192), ("qkv", 3840, 2560, 8192)]


@pytest.mark.parametrize("name,M,K,n", CASES)
def test_prefill_gemm_accumulators_bitexact(name, M, K, n):
    torch = need_cuda()
    L = synth().layer(80_000 + M + K + n, M, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M)
    q_np = np.random.default_rng(M + n).integers(-127, 128, (n, K), dtype=np.int8)
    q = torch.from_numpy(q_np).cuda()
    qs = torch.from_numpy(q_np.astype(np.int64).sum(1).astype(np.int32)).cuda()
    got = layer.acc(q, qs).cpu().numpy()
    want = orc.ternary_acc_omp(L.packed, q_np, M, K)
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} accumulators differ, first (token, row) {bad[:4].tolist()}"
    layer.close()
    obn().check_device_errors()


@pytest.mark.parametrize("name,M,K,n", CASES)
def test_prefill_forward_matches_oracle(name, M, K, n):
    torch = need_cuda()
    L = synth().layer(81_000 + M + K + n, M, K)
    x = synth().activations(82_000 + n + K, n, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    xd = torch.from_numpy(x).cuda()
    y = layer.forward(xd).cpu().numpy()
    q_gpu, s_gpu, qs_gpu = obn().rmsnorm_quantize(xd, torch.from_numpy(L.gamma).cuda())
    # oracle: rmsnorm.wgsl -> quantize.wgsl -> integer core -> the GEMM epilogue
    q_ref, s_ref = orc.quantize(orc.rmsnorm(x, L.gamma))
    assert np.array_equal(q_gpu.cpu().numpy(), q_ref)
    assert np.array_equal(s_gpu.cpu().numpy(), s_ref)
    assert np.array_equal(qs_gpu.cpu().numpy(), q_ref.astype(np.int64).sum(1).astype(np.int32))
    acc = orc.ternary_acc_omp(L.packed, q_ref, M, K)
    scale = L.row_scales()[None, :] * s_ref[:, None]          # f32 products, rounded once
    want = acc.astype(np.float32) * scale
    assert want.dtype == np.float32
    assert np.array_equal(y, want), float(np.abs(y - want).max())
    np.testing.assert_allclose(y, want, rtol=1e-5, atol=0)  # the north-star bound, stated
    layer.close()
    obn().check_device_errors()
