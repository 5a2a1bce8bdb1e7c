"""GPU parity: libobn.so's sm_100a kernels against the CPU oracle and golden fixtures.

Bar (from the north star): int8 activations, per-token scales and int32
accumulators bit-exact; float32 outputs within 1e-5 relative. The kernels are
built to round exactly like the oracle, so float outputs are also checked for
bit equality, with the 1e-5 bound asserted as the contract in addition.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle as orc
from _util import GOLDEN, need_cuda, obn, synth

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # north_star: scaled fp32 outputs within 1e-5 relative


@pytest.fixture(scope="module")
def torch():
    return need_cuda()


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layer_from(torch, L, norm=True):
    return obn().BitLinear.from_i2s(L.blob(), L.K, L.M, norm_weight=L.gamma if norm else None)


def assert_fp_parity(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    rel = np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want.astype(np.float64)), 1e-30)
    assert (rel <= RTOL).all(), f"max rel err {rel.max()}"
    assert np.array_equal(got, want), "float outputs differ from the oracle's rounding"


# ------------------------------------------------------------------- repack
@pytest.mark.parametrize("M,K", [(1, 128), (17, 256), (300, 384), (2560, 2560), (3840, 2560),
                                 (6912, 2560), (2560, 6912)])
def test_repack_round_trip(torch, M, K):
    L = synth().layer(M * 7 + K, M, K)
    layer = layer_from(torch, L)
    back = layer.export_i2s().cpu().numpy()
    assert np.array_equal(back, L.packed)


def test_create_from_device_buffers_matches_load(torch):
    L = synth().layer(5, 384, 512)
    packed = to_dev(torch, L.packed.reshape(-1).view(np.uint32))  # [M, K/16] u32 like the reference
    scales = to_dev(torch, L.row_scales())
    gamma = to_dev(torch, L.gamma)
    a = obn().BitLinear(packed, scales, gamma, 512, 384)
    b = layer_from(torch, L)
    x = to_dev(torch, synth().activations(6, 3, 512))
    assert torch.equal(a.forward(x), b.forward(x))
    assert np.array_equal(a.export_i2s().cpu().numpy(), L.packed)


# ------------------------------------------------------------------- RMSNorm + quantize
@pytest.mark.parametrize("K", [128, 256, 2560, 6912, 9216])
@pytest.mark.parametrize("n", [1, 5, 64])
@pytest.mark.parametrize("norm", [True, False])
def test_rmsnorm_quantize_bitexact(torch, K, n, norm):
    x = synth().activations(K + n, n, K)
    gamma = synth().layer(K, 1, K).gamma
    q, s, qs = obn().rmsnorm_quantize(to_dev(torch, x), to_dev(torch, gamma) if norm else None)
    src = orc.rmsnorm(x, gamma, 1e-5) if norm else x
    q_ref, s_ref = orc.quantize(src)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(qs.cpu().numpy(), q_ref.astype(np.int64).sum(1))


@pytest.mark.parametrize("K", [128, 640, 2560, 4100, 6912, 7936, 9216])
@pytest.mark.parametrize("n", [257, 1000, 3001])
@pytest.mark.parametrize("norm", [True, False])
def test_rmsnorm_quantize_many_tokens_bitexact(torch, K, n, norm):
    # above 256 tokens the quantize pass runs 64 threads per token, four tokens per
    # CTA, each slot's next row staged by a bulk copy: ragged token counts leave
    # slots of the last CTAs idle, and K = 640 leaves the last column quad to the
    # first half of the slot's threads. Rows of 4097 .. 7936 columns take the
    # 128-thread form (three double-buffered groups per CTA): K = 4100 ends on a
    # partial column pair sweep, 7936 fills its shared memory; K = 9216 is past it
    x = synth().activations(3 * K + n, n, K)
    x[n // 2] = 0.0                                       # an all-zero row: scale 1, q 0
    gamma = (synth().layer(K + 1, 1, K).gamma if K % 128 == 0 else
             (1 + 0.1 * np.random.default_rng(K).standard_normal(K)).astype(np.float32))
    q, s, qs = obn().rmsnorm_quantize(to_dev(torch, x), to_dev(torch, gamma) if norm else None)
    src = orc.rmsnorm(x, gamma, 1e-5) if norm else x
    q_ref, s_ref = orc.quantize(src)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(qs.cpu().numpy(), q_ref.astype(np.int64).sum(1))


@pytest.mark.parametrize("K", [4, 128, 2560, 6912])
def test_rmsnorm_bitexact(torch, K):
    x = synth().activations(K, 3, K)
    gamma = (1 + 0.1 * np.random.default_rng(K).standard_normal(K)).astype(np.float32)
    y = obn().rmsnorm(to_dev(torch, x), to_dev(torch, gamma)).cpu().numpy()
    assert np.array_equal(y, orc.rmsnorm(x, gamma, 1e-5))


def test_quantize_edge_cases(torch):
    K = 256
    rows = np.zeros((6, K), np.float32)
    rows[1, 17] = -3.5                                   # single nonzero, negative absmax
    rows[2, :] = np.arange(K, dtype=np.float32) - 128.0  # ties: x*127/128 hits .5 boundaries
    rows[2, 0] = -127.0 * 1.0078125                      # make absmax exact for the ties
    rows[3, :] = 1e30                                    # huge, constant
    rows[4, ::2] = 1e-30                                 # tiny
    rows[5, :] = (np.arange(K) % 3 - 1) * 0.5            # many exact .5-multiples
    q, s, qs = obn().rmsnorm_quantize(to_dev(torch, rows))
    q_ref, s_ref = orc.quantize(rows)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert s_ref[0] == 1.0 and not q_ref[0].any()       # zero row: scale 1, q 0
    assert np.array_equal(qs.cpu().numpy(), q_ref.astype(np.int64).sum(1))


def test_quantize_ties_round_to_even_on_gpu(torch):
    x = np.array([[127.0, -63.5, 2.5, 0.5, -0.5, 1.5, -2.5, 3.5]], np.float32)
    q, _, _ = obn().rmsnorm_quantize(to_dev(torch, x))
    assert q.cpu().numpy()[0].tolist() == [127, -64, 2, 0, 0, 2, -2, 4]


# ------------------------------------------------------------------- integer core
@pytest.mark.parametrize("M,K", [(8, 256), (300, 384), (2560, 2560), (3840, 2560),
                                 (6912, 2560), (2560, 6912)])
@pytest.mark.parametrize("n", [1, 2, 3, 7, 8, 9, 16, 64])
def test_int32_accumulators_bitexact(torch, M, K, n):
    L = synth().layer(M + K + n, M, K)
    layer = layer_from(torch, L, norm=False)
    q_np = np.random.default_rng(n).integers(-127, 128, (n, K), dtype=np.int8)
    q = to_dev(torch, q_np)
    qs = to_dev(torch, q_np.astype(np.int64).sum(1).astype(np.int32))
    acc = layer.acc(q, qs).cpu().numpy()
    assert np.array_equal(acc, orc.ternary_acc(L.packed, q_np, M, K))


def test_int32_extremes(torch):
    # every code at its extremes: all +1 rows, all -1 rows, the unused code 3
    # (decodes to +2 in the shader formula) and q = +-127 everywhere.
    K, M = 6912, 4
    packed = np.empty((M, K // 4), np.uint8)
    packed[0] = 0xAA
    packed[1] = 0x00
    packed[2] = 0xFF
    packed[3] = 0x55
    blob = obn().i2s.make_tensor(packed, 1.0)
    layer = obn().BitLinear.from_i2s(blob, K, M)
    for val in (127, -127):
        q_np = np.full((2, K), val, np.int8)
        acc = layer.acc(to_dev(torch, q_np),
                        to_dev(torch, q_np.astype(np.int64).sum(1).astype(np.int32))).cpu().numpy()
        assert np.array_equal(acc, orc.ternary_acc(packed, q_np, M, K))
        assert acc[0, 0] == val * K and acc[0, 1] == -val * K and acc[0, 2] == 2 * val * K


# ------------------------------------------------------------------- BitLinear forward
@pytest.mark.parametrize("shape", list(synth().SHAPES_2B))
@pytest.mark.parametrize("n", [1, 8])
def test_forward_matches_oracle_2b_shapes(torch, shape, n):
    M, K = synth().SHAPES_2B[shape]
    L = synth().layer(list(synth().SHAPES_2B).index(shape) * 100 + n, M, K)
    x = synth().activations(n * 31 + M, n, K)
    layer = layer_from(torch, L)
    y = layer.forward(to_dev(torch, x)).cpu().numpy()
    y_ref, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)
    assert_fp_parity(y, y_ref)


@pytest.mark.parametrize("n", [2, 32, 64, 100])
def test_forward_batched(torch, n):
    M, K = 2560, 2560
    L = synth().layer(n, M, K)
    x = synth().activations(n + 1, n, K)
    y = layer_from(torch, L).forward(to_dev(torch, x)).cpu().numpy()
    y_ref, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)
    assert_fp_parity(y, y_ref)


def test_forward_without_norm_and_odd_rows(torch):
    M, K = 1000, 384
    L = synth().layer(3, M, K)
    for n in (1, 3):
        x = synth().activations(4 + n, n, K)
        y = layer_from(torch, L, norm=False).forward(to_dev(torch, x)).cpu().numpy()
        y_ref, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K)
        assert_fp_parity(y, y_ref)


def test_forward_on_side_stream_and_repeatable(torch):
    M, K = 3840, 2560
    L = synth().layer(11, M, K)
    layer = layer_from(torch, L)
    x = to_dev(torch, synth().activations(12, 4, K))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = layer.forward(x)
        b = layer.forward(x)
    s.synchronize()
    assert torch.equal(a, b)
    y_ref, _, _ = orc.bitlinear(x.cpu().numpy(), L.packed, L.row_scales(), M, K, norm_w=L.gamma)
    assert_fp_parity(a.cpu().numpy(), y_ref)


def test_chained_forwards_keep_stream_order(torch):
    # y1 = L1(x); y2 = L2(y1): the second call's quantize must see the first's output.
    K = 2560
    L1 = synth().layer(21, K, K)
    L2 = synth().layer(22, K, K)
    l1, l2 = layer_from(torch, L1), layer_from(torch, L2)
    x = synth().activations(23, 2, K)
    for _ in range(3):
        y2 = l2.forward(l1.forward(to_dev(torch, x))).cpu().numpy()
    r1, _, _ = orc.bitlinear(x, L1.packed, L1.row_scales(), K, K, norm_w=L1.gamma)
    r2, _, _ = orc.bitlinear(r1, L2.packed, L2.row_scales(), K, K, norm_w=L2.gamma)
    assert_fp_parity(y2, r2)


def test_weight_scale_linearity_full_size(torch):
    # Doubling the weight scale doubles every output exactly (x2 is exact in fp32).
    M, K = 6912, 2560
    L = synth().layer(31, M, K)
    x = to_dev(torch, synth().activations(32, 8, K))
    a = layer_from(torch, L).forward(x)
    L.scale *= 2.0
    b = layer_from(torch, L).forward(x)
    assert torch.equal(b, a * 2)


def test_gemv_and_gemm_orders_agree_within_tolerance(torch):
    # n == 1 rounds (acc*s_w)*s_x, n > 1 acc*(s_w*s_x): one token repeated twice
    # must agree with the single-token call to 1e-5 relative.
    M, K = 2560, 2560
    L = synth().layer(41, M, K)
    layer = layer_from(torch, L)
    x1 = synth().activations(42, 1, K)
    a = layer.forward(to_dev(torch, x1)).cpu().numpy()[0]
    b = layer.forward(to_dev(torch, np.repeat(x1, 2, 0))).cpu().numpy()
    assert np.array_equal(b[0], b[1])
    np.testing.assert_allclose(a, b[0], rtol=RTOL, atol=1e-6)


# ------------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", ["cfg0_fused_gemv", "cfg1_o_b8", "cfg1_down_b3_nonorm"])
def test_golden_seeded_configs(torch, name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    seed, n, M, K, norm = (int(g["seed"]), int(g["n"]), int(g["M"]), int(g["K"]), bool(g["norm"]))
    L = synth().layer(seed, M, K)
    x = to_dev(torch, synth().activations(seed + 1, n, K))
    layer = layer_from(torch, L, norm=norm)
    assert_fp_parity(layer.forward(x).cpu().numpy(), g["y"])
    q, s, qs = obn().rmsnorm_quantize(x, to_dev(torch, L.gamma) if norm else None)
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(s.cpu().numpy(), g["scales"])
    assert np.array_equal(qs.cpu().numpy(), g["qsum"])
    assert np.array_equal(layer.acc(q, qs).cpu().numpy(), g["acc"])


def test_golden_reference_kat_gemv(torch):
    # ternary-gemv.test.ts:13-33 inputs (mulberry32 seed 42), M=8, K=256.
    g = np.load(os.path.join(GOLDEN, "kat_gemv_seed42.npz"))
    s_w = g["s_w"]
    layer = obn().BitLinear(to_dev(torch, g["packed"]), to_dev(torch, s_w), None, 256, 8)
    q = to_dev(torch, g["q"][None])
    qs = to_dev(torch, np.array([g["q"].astype(np.int64).sum()], np.int32))
    sx = to_dev(torch, np.array([g["s_x"]], np.float32))
    assert np.array_equal(layer.acc(q, qs).cpu().numpy(), g["acc"])
    assert_fp_parity(layer.matmul(q, sx, qs).cpu().numpy()[0], g["y"])


def test_golden_reference_kat_gemm_layout(torch):
    # ternary-gemm.test.ts:37-72: M=4, K=128, N=3, per-token scales.
    g = np.load(os.path.join(GOLDEN, "kat_gemm_layout.npz"))
    layer = obn().BitLinear(to_dev(torch, g["packed"]), to_dev(torch, g["s_w"]), None, 128, 4)
    q = to_dev(torch, g["q"])
    qs = to_dev(torch, g["q"].astype(np.int64).sum(1).astype(np.int32))
    assert_fp_parity(layer.matmul(q, to_dev(torch, g["s_x"]), qs).cpu().numpy(), g["y"])


def test_golden_reference_kat_e2e(torch):
    # bitlinear-e2e.test.ts:111-139: randf32(256, 10) through a 128x256 layer, n = 1.
    g = np.load(os.path.join(GOLDEN, "kat_e2e_n1.npz"))
    layer = obn().BitLinear(to_dev(torch, g["packed"]), to_dev(torch, np.ones(128, np.float32)),
                            None, 256, 128)
    assert_fp_parity(layer.forward(to_dev(torch, g["x"])).cpu().numpy(), g["y"])


@pytest.mark.parametrize("val,expect", [(1, 128.0), (-1, -128.0), (0, 0.0)])
def test_reference_known_answers_on_gpu(torch, val, expect):
    # ternary-gemv.test.ts:35-64 (rows of all +1 / -1 / 0 against ones -> +-128 / 0)
    # and bitlinear-e2e.test.ts:192-217 (constant 0.5 through all +1, K=256 -> 128).
    K = 128
    packed = obn().i2s.pack_rows(np.full((1, K), val, np.int8))
    layer = obn().BitLinear.from_i2s(obn().i2s.make_tensor(packed, 1.0), K, 1)
    q = torch.ones((1, K), dtype=torch.int8, device="cuda")
    qs = torch.tensor([K], dtype=torch.int32, device="cuda")
    y = layer.matmul(q, torch.ones(1, device="cuda"), qs).item()
    assert y == expect
    K = 256
    packed = obn().i2s.pack_rows(np.ones((1, K), np.int8))
    layer = obn().BitLinear.from_i2s(obn().i2s.make_tensor(packed, 1.0), K, 1)
    y = layer.forward(torch.full((1, K), 0.5, device="cuda")).item()
    assert abs(y - 128.0) < 0.5


# ------------------------------------------------------------------- errors
def test_error_paths_on_gpu(torch):
    lib = obn().lib()
    L = synth().layer(1, 256, 256)
    layer = layer_from(torch, L)
    x = to_dev(torch, synth().activations(2, 2, 256))
    y = torch.empty((2, 256), device="cuda")
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    rc = lib.obn_bitlinear_forward(layer.handle, ctypes.c_void_p(x.data_ptr()), 2,
                                   ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(small.data_ptr()),
                                   16, None)
    assert rc == obn()._lib.OBN_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.obn_error_message()
    ws = torch.empty(layer.workspace_bytes(2) + 256, dtype=torch.uint8, device="cuda")
    rc = lib.obn_bitlinear_forward(layer.handle, ctypes.c_void_p(x.data_ptr() + 4), 2,
                                   ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                   ws.numel(), None)
    assert rc == obn()._lib.OBN_ERR_INVALID_ARGUMENT
    with pytest.raises(obn().ObnError):
        obn().BitLinear.from_i2s(L.blob()[:100], 256, 256)


def test_no_device_wait_gave_up(torch):
    torch.cuda.synchronize()
    obn().check_device_errors()


@pytest.mark.parametrize("M,K,n", [(2560, 2560, 1), (2560, 6912, 3), (2560, 2560, 8),
                                   (2560, 6912, 64), (3000, 512, 300),
                                   # CTA-pair tiles (from 512 tokens), full and partial
                                   (2560, 2560, 512), (3000, 512, 777)])
def test_forward_residual_is_forward_plus_add(M, K, n):
    # y += forward(x) in the epilogue equals forward(x) then the f32 add, bit for bit
    torch = need_cuda()
    L = synth().layer(M + K + n, M, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    x = torch.from_numpy(synth().activations(n + 1, n, K)).cuda()
    y0 = torch.from_numpy(synth().activations(n + 2, n, M)).cuda()
    want = (y0 + layer.forward(x)).cpu().numpy()
    y = y0.clone()
    layer.forward_residual(x, y)
    assert np.array_equal(y.cpu().numpy(), want)
