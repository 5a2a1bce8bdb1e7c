"""GPU parity of the merged gate|up FFN layer (obn_bitlinear_load_i2s_gated).

forward(x) must equal, bit for bit, the reference's FFN::forward_gated front:
two BitLinear forwards (gate, up) on the same input followed by ReLU^2 on gate
and an elementwise multiply by up (oracle: bitlinear twice + relu2_mul), for
every matmul path: the fused single-token kernel, the dp4a GEMV, the split-K
and persistent tensor-core GEMMs (whose epilogues form act(gate) * up). The interleaved rows are also checked through
the exact accumulators.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu


def layers(M, K, seed):
    gate = synth().layer(seed, M, K)
    up = synth().layer(seed + 1, M, K)
    return gate, up


@pytest.mark.parametrize("M,K,n", [(6912, 2560, 1), (6912, 2560, 2), (6912, 2560, 8),
                                   (6912, 2560, 64), (1000, 384, 3), (300, 256, 40),
                                   (6912, 2560, 300), (513, 640, 17),
                                   # split-K over 3 and 7 CTAs (owner row blocks 44, 20)
                                   (2560, 2560, 4), (1280, 2560, 9), (1280, 2560, 40),
                                   # CTA-pair tiles (from 512 tokens), full and partial;
                                   # the last wave split into half tiles (6912 x 512),
                                   # every tile split, the last half partial (640 x 700)
                                   (6912, 2560, 512), (513, 640, 600), (640, 640, 700)])
def test_gated_forward_matches_two_bitlinears(M, K, n):
    torch = need_cuda()
    gate, up = layers(M, K, 100 + n)
    L = obn().BitLinear.from_i2s_gated(gate.blob(), up.blob(), K, M, norm_weight=gate.gamma)
    assert (L.out_dim, L.rows) == (M, 2 * M)
    x = synth().activations(200 + n, n, K)
    y = L.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    g, _, _ = orc.bitlinear(x, gate.packed, gate.row_scales(), M, K, norm_w=gate.gamma)
    u, _, _ = orc.bitlinear(x, up.packed, up.row_scales(), M, K, norm_w=gate.gamma)
    assert np.array_equal(y, orc.relu2_mul(g, u))
    L.close()


@pytest.mark.parametrize("M,K,n", [(6912, 2560, 1), (6912, 2560, 2), (6912, 2560, 64),
                                   (300, 256, 3), (6912, 2560, 300), (513, 640, 17),
                                   (1280, 2560, 9), (513, 640, 600), (640, 640, 700)])
def test_gated_silu_forward(M, K, n):
    """SiLU gate (x / (1 + exp(-x)), activation.wgsl): every matmul path within the
    error of the device's expf (a few ulp) of silu(gate) * up."""
    torch = need_cuda()
    gate, up = layers(M, K, 300 + n)
    L = obn().BitLinear.from_i2s_gated(gate.blob(), up.blob(), K, M, norm_weight=gate.gamma)
    L.set_activation(1)
    x = synth().activations(400 + n, n, K)
    y = L.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    g, _, _ = orc.bitlinear(x, gate.packed, gate.row_scales(), M, K, norm_w=gate.gamma)
    u, _, _ = orc.bitlinear(x, up.packed, up.row_scales(), M, K, norm_w=gate.gamma)
    with np.errstate(over="ignore"):
        want = (g / (np.float32(1) + np.exp(-g))).astype(np.float32) * u
    np.testing.assert_allclose(y, want, rtol=1e-6, atol=1e-30)
    L.close()


def test_gated_rows_interleave():
    torch = need_cuda()
    M, K, n = 300, 256, 20
    gate, up = layers(M, K, 5)
    L = obn().BitLinear.from_i2s_gated(gate.blob(), up.blob(), K, M)
    q = np.random.default_rng(3).integers(-127, 128, (n, K), dtype=np.int8)
    qs = q.astype(np.int64).sum(1).astype(np.int32)
    acc = L.acc(torch.from_numpy(q).cuda(), torch.from_numpy(qs).cuda()).cpu().numpy()
    assert np.array_equal(acc[:, 0::2], orc.ternary_acc(gate.packed, q, M, K))
    assert np.array_equal(acc[:, 1::2], orc.ternary_acc(up.packed, q, M, K))
    rows = L.export_i2s().cpu().numpy()
    assert np.array_equal(rows[0::2], gate.packed) and np.array_equal(rows[1::2], up.packed)
    L.close()
    obn().check_device_errors()
