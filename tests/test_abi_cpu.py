"""CPU-only checks of the C ABI library and the host-side logic.

No kernel runs here: the library is loaded, its exports are compared with the
declarations in include/obn.h, and the host-side validation / error paths are
exercised (on a machine without a GPU, device work reports OBN_ERR_NO_DEVICE).
"""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle as orc
from _util import GOLDEN, ROOT, obn, sha256, synth

HEADER = os.path.join(ROOT, "include", "obn.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"OBN_API\s+[\w\s\*]+?\b(obn_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = obn().lib()
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/obn.h but not exported"
    # and the Python binding covers exactly the declared surface
    assert sorted(obn()._lib.SIGNATURES) == syms


def test_version_and_no_error_initially():
    lib = obn().lib()
    assert lib.obn_version() == 100
    lib.obn_bitlinear_workspace_bytes(None, 1)
    assert lib.obn_error_message() is None or isinstance(lib.obn_error_message(), bytes)


def test_null_arguments_are_rejected_with_a_message():
    lib = obn().lib()
    h = ctypes.c_void_p()
    rc = lib.obn_bitlinear_load_i2s(None, 0, 128, 4, None, 1e-5, 0, ctypes.byref(h))
    assert rc == obn()._lib.OBN_ERR_INVALID_ARGUMENT
    assert b"null" in lib.obn_error_message()
    assert lib.obn_bitlinear_forward(None, None, 1, None, None, 0, None) == \
        obn()._lib.OBN_ERR_INVALID_ARGUMENT


def test_non_block_aligned_in_dim_is_unsupported():
    lib = obn().lib()
    blob = np.zeros(200 * 4 // 4 + 32, np.uint8)
    h = ctypes.c_void_p()
    rc = lib.obn_bitlinear_load_i2s(blob.ctypes.data, blob.size, 200, 4, None, 1e-5, 0,
                                    ctypes.byref(h))
    assert rc == obn()._lib.OBN_ERR_UNSUPPORTED
    assert b"multiple of 128" in lib.obn_error_message()


def test_short_tensor_is_rejected():
    lib = obn().lib()
    blob = np.zeros(128 * 4 // 4 + 16, np.uint8)  # trailer shorter than 32 bytes
    h = ctypes.c_void_p()
    rc = lib.obn_bitlinear_load_i2s(blob.ctypes.data, blob.size, 128, 4, None, 1e-5, 0,
                                    ctypes.byref(h))
    assert rc == obn()._lib.OBN_ERR_INVALID_ARGUMENT


def test_error_message_is_thread_local():
    import threading
    lib = obn().lib()
    h = ctypes.c_void_p()
    lib.obn_bitlinear_load_i2s(None, 0, 128, 4, None, 1e-5, 0, ctypes.byref(h))
    seen = []

    def other():
        seen.append(lib.obn_error_message())
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [None]
    assert lib.obn_error_message() is not None


def test_no_device_is_reported_not_hidden():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = obn().lib()
    L = synth().layer(1, 4, 128)
    blob = L.blob()
    h = ctypes.c_void_p()
    rc = lib.obn_bitlinear_load_i2s(blob.ctypes.data, blob.size, 128, 4, None, 1e-5, 0,
                                    ctypes.byref(h))
    assert rc == obn()._lib.OBN_ERR_NO_DEVICE
    assert h.value is None


def test_workspace_size_formula():
    lib = obn().lib()
    assert lib.obn_bitlinear_workspace_bytes(None, 4) == 0


# ---------------------------------------------------------------- host I2_S logic
@pytest.mark.parametrize("M,K,seed", [(1, 128, 1), (7, 256, 2), (33, 2560, 3)])
def test_numpy_packer_matches_oracle(M, K, seed):
    v = orc.rand_ternary(M * K, seed).reshape(M, K)
    p = obn().i2s.pack_rows(v)
    assert np.array_equal(p, orc.i2s_pack_matrix(v))
    assert np.array_equal(obn().i2s.unpack_rows(p, K), v)


def test_tensor_blob_round_trip():
    i2s = obn().i2s
    v = orc.rand_ternary(8 * 256, 5).reshape(8, 256)
    blob = i2s.make_tensor(i2s.pack_rows(v), 1.75)
    assert blob.size == 8 * 256 // 4 + 32
    packed, scale = i2s.split_tensor(blob, 256, 8)
    assert scale == 1.75 and np.array_equal(i2s.unpack_rows(packed, 256), v)
    # the trailer replicates the scale 8 times (loader.rs reads the first one)
    assert np.all(blob[-32:].view("<f4") == np.float32(1.75))


def test_synthetic_distribution():
    L = synth().layer(0, 512, 2560)
    w = obn().i2s.unpack_rows(L.packed, 2560)
    frac = [(w == v).mean() for v in (-1, 0, 1)]
    assert abs(frac[0] - 0.3) < 0.01 and abs(frac[1] - 0.4) < 0.01 and abs(frac[2] - 0.3) < 0.01
    assert 0.5 <= L.scale <= 2.0


@pytest.mark.parametrize("name", ["cfg0_fused_gemv", "cfg1_o_b8", "cfg1_down_b3_nonorm"])
def test_golden_fixtures_match_oracle(name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    seed, n, M, K, norm = (int(g["seed"]), int(g["n"]), int(g["M"]), int(g["K"]), bool(g["norm"]))
    L = synth().layer(seed, M, K)
    x = synth().activations(seed + 1, n, K)
    assert sha256(L.packed, np.float32(L.scale), L.gamma, x) == str(g["inputs_sha"])
    y, q, s = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma if norm else None)
    assert np.array_equal(q, g["q"]) and np.array_equal(s, g["scales"])
    assert np.array_equal(y, g["y"])
    assert np.array_equal(orc.ternary_acc(L.packed, q, M, K), g["acc"])


def test_golden_kat_fixtures_match_oracle():
    g = np.load(os.path.join(GOLDEN, "kat_gemv_seed42.npz"))
    y = orc.ternary_gemv(g["packed"], g["q"], g["s_w"], g["s_x"], 8, 256)
    assert np.array_equal(y, g["y"])
    g = np.load(os.path.join(GOLDEN, "kat_gemm_layout.npz"))
    assert np.array_equal(orc.ternary_gemm(g["packed"], g["q"], g["s_w"], g["s_x"], 4, 128), g["y"])
