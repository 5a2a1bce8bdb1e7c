"""GPU parity of the tensor-core (tcgen05 kind::i8) ternary GEMM path.

Token counts >= 16 run on the tensor cores, and so do 4-15 tokens when the
layer has few enough 128-row tiles for the split-K (cluster) form. Shapes cover
partial tiles in both the weight-row (128) and token (16/32/64/128/256)
dimensions, single and many K blocks, one and several tiles per persistent CTA,
cluster sizes 2 through 8, and the CTA-pair kernel's half-width (128-token)
units, with the last half ragged.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return need_cuda()


def run_acc(torch, M, K, n, seed):
    L = synth().layer(seed, M, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M)
    q_np = np.random.default_rng(seed + 1).integers(-127, 128, (n, K), dtype=np.int8)
    q = torch.from_numpy(q_np).cuda()
    qs = torch.from_numpy(q_np.astype(np.int64).sum(1).astype(np.int32)).cuda()
    acc = layer.acc(q, qs).cpu().numpy()
    return acc, orc.ternary_acc(L.packed, q_np, M, K)


@pytest.mark.parametrize("M,K,n", [(128, 128, 16), (128, 256, 32), (256, 384, 64)])
def test_gemm_small_exact(torch, M, K, n):
    got, want = run_acc(torch, M, K, n, M + K + n)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("M,K,n", [(1, 128, 16), (100, 256, 17), (129, 128, 33), (300, 384, 100),
                                   (513, 640, 129), (1000, 256, 257), (2560, 2560, 64),
                                   (6912, 2560, 32), (2560, 6912, 64), (3840, 2560, 300),
                                   (128, 256, 200), (129, 128, 300), (384, 640, 513),
                                   # CTA pairs with half-width units: every tile split,
                                   # the last half partial (1280 x 900); the last partial
                                   # wave split (2560 x 2048: 80 tiles on 74 pairs)
                                   (1280, 640, 900), (2560, 384, 2048), (2560, 256, 8092)])
def test_gemm_acc_bitexact(torch, M, K, n):
    got, want = run_acc(torch, M, K, n, M * 3 + K + n)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [4, 8, 16, 32, 64, 512, 2048])
def test_gemm_forward_matches_oracle(torch, n):
    M, K = 2560, 2560
    L = synth().layer(700 + n, M, K)
    x = synth().activations(701 + n, n, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    y = layer.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    y_ref, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)
    assert np.array_equal(y, y_ref)


@pytest.mark.parametrize("M,K,n", [(128, 2560, 16), (300, 2560, 64), (2560, 2560, 32),
                                   (3840, 2560, 128), (6912, 2560, 100), (2560, 6912, 64),
                                   (1000, 384, 48), (640, 1280, 128), (2560, 9216, 16),
                                   (2000, 640, 20), (1920, 1664, 40), (2560, 2560, 4),
                                   (3840, 2560, 8), (2560, 6912, 12), (6912, 2560, 5)])
def test_gemm_split_k_cluster_bitexact(torch, M, K, n):
    # token counts <= 128 with few 128-row tiles run split-K over a cluster of up
    # to 8 CTAs (bulk-copy reduce-scatter through distributed shared memory);
    # these shapes reach cluster sizes 2 through 8, including ragged row splits
    got, want = run_acc(torch, M, K, n, M + 7 * K + n)
    assert np.array_equal(got, want)


def test_gemm_many_tiles_per_cta(torch):
    # 54 row tiles x 8 token tiles = 432 tiles over <= 148 persistent CTAs.
    M, K, n = 6912, 256, 2048
    got, want = run_acc(torch, M, K, n, 9)
    assert np.array_equal(got, want)


def test_gemm_device_errors_clean(torch):
    torch.cuda.synchronize()
    obn().check_device_errors()
