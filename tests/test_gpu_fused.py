"""GPU parity of the fused few-token BitLinear kernel (k_bitlinear_mma).

For 2..8 tokens on layers with at least 8192 weight rows and in_dim <= 3072,
one kernel normalises (rmsnorm.wgsl), quantizes (quantize.wgsl) and multiplies
(ternary_gemm.wgsl) with every CTA redoing the per-token reductions: one warp
per token, the shader's halving tree mapped onto local adds and shuffles. Each
case compares the forward with the oracle's BitLinear bit for bit, with and
without the RMSNorm, for in_dim not a multiple of 256 (the last column quads
fall to the first half of the warp), and for the residual form (y += forward).
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return need_cuda()


@pytest.mark.parametrize("M,K", [(8192, 128), (8200, 640), (9000, 2560), (8192, 3072)])
@pytest.mark.parametrize("n", [2, 5, 8])
@pytest.mark.parametrize("norm", [True, False])
def test_fused_forward_bitexact(torch, M, K, n, norm):
    L = synth().layer(60_000 + M + K + n, M, K)
    x = synth().activations(61_000 + K + n, n, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma if norm else None)
    y = layer.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    want = orc.bitlinear_omp(x, L.packed, L.row_scales(), M, K,
                             norm_w=L.gamma if norm else None)
    assert np.array_equal(y, want), float(np.abs(y - want).max())
    layer.close()


@pytest.mark.parametrize("n", [3, 8])
def test_fused_residual_forward_bitexact(torch, n):
    M, K = 8192, 2560
    L = synth().layer(62_000 + n, M, K)
    x = synth().activations(63_000 + n, n, K)
    base = synth().activations(64_000 + n, n, M)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    y = torch.from_numpy(base.copy()).cuda()
    layer.forward_residual(torch.from_numpy(x).cuda(), y)
    got = y.cpu().numpy()
    want = (base + orc.bitlinear_omp(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)).astype(
        np.float32)
    assert np.array_equal(got, want)
    layer.close()
    obn().check_device_errors()
