"""ctypes binding of libobn.so (the C ABI declared in include/obn.h).

The shared library is built in-tree by ``0xbitnet_b200/csrc/Makefile``
(``python __graft_entry__.py build``). There is no fallback: if the library is
missing, importing the package raises, so nothing can silently run elsewhere.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libobn.so")

OBN_OK = 0
OBN_ERR_INVALID_ARGUMENT = -1
OBN_ERR_UNSUPPORTED = -2
OBN_ERR_CUDA = -3
OBN_ERR_OUT_OF_MEMORY = -4
OBN_ERR_DEVICE_TIMEOUT = -5
OBN_ERR_NO_DEVICE = -6

# Every symbol include/obn.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES = {
    "obn_version": (_I, []),
    "obn_error_message": (ctypes.c_char_p, []),
    "obn_bitlinear_load_i2s": (_I, [_P, _SZ, _I, _I, _P, _F, _I, ctypes.POINTER(_P)]),
    "obn_bitlinear_create": (_I, [_P, _P, _P, _F, _I, _I, _P, ctypes.POINTER(_P)]),
    "obn_bitlinear_free": (None, [_P]),
    "obn_bitlinear_in_dim": (_I, [_P]),
    "obn_bitlinear_out_dim": (_I, [_P]),
    "obn_bitlinear_rows": (_I, [_P]),
    "obn_bitlinear_create_gated": (_I, [_P, _P, _P, _P, _P, _F, _I, _I, _P, ctypes.POINTER(_P)]),
    "obn_bitlinear_load_i2s_gated": (_I, [_P, _SZ, _P, _SZ, _I, _I, _P, _F, _I, ctypes.POINTER(_P)]),
    "obn_bitlinear_load_i2s_concat": (_I, [_I, _P, _P, _P, _I, _P, _F, _I, ctypes.POINTER(_P)]),
    "obn_bitlinear_set_activation": (_I, [_P, _I]),
    "obn_activation": (_I, [_P, _SZ, _I, _P, _P]),
    "obn_bitlinear_workspace_bytes": (_SZ, [_P, _I]),
    "obn_bitlinear_forward": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "obn_bitlinear_forward_noalloc": (_I, [_P, _P, _I, _P, _P]),
    "obn_measure_mma_rate": (_I, [_I, _I, _I, ctypes.POINTER(ctypes.c_double)]),
    "obn_bitlinear_forward_residual": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "obn_bitlinear_forward_tp": (_I, [_P, _P, _I, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "obn_lm_head_f16": (_I, [_P, _I, _I, _P, _P, _F, _I, _P, _P]),
    "obn_lm_head_workspace_bytes": (_SZ, [_I, _I]),
    "obn_lm_head_f16_batched": (_I, [_P, _I, _I, _P, _P, _F, _I, _P, _P, _SZ, _P]),
    "obn_rope_kv_append": (_I, [_P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _P]),
    "obn_attention_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "obn_attention_decode": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _SZ, _P]),
    "obn_rope_kv_append_at": (_I, [_P, _I, _I, _I, _I, _I, _P, _F, _P, _P, _P, _I, _P]),
    "obn_attention_decode_at": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _F, _P, _P, _SZ,
                                     _P]),
    "obn_attention_decode_rope": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _F, _P, _P, _SZ,
                                       _P]),
    "obn_attention_decode_rope_at": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _F, _F, _P, _P,
                                          _SZ, _P]),
    "obn_add": (_I, [_P, _P, _SZ, _P, _P]),
    "obn_embed_f16": (_I, [_P, _I, _I, _P, _I, _P, _P]),
    "obn_rmsnorm_quantize": (_I, [_P, _P, _F, _I, _I, _P, _P, _P, _P]),
    "obn_rmsnorm": (_I, [_P, _P, _F, _I, _I, _P, _P]),
    "obn_ternary_matmul": (_I, [_P, _P, _P, _P, _I, _P, _P]),
    "obn_ternary_acc": (_I, [_P, _P, _P, _I, _P, _P]),
    "obn_bitlinear_export_i2s": (_I, [_P, _P, _P]),
    "obn_check_device_errors": (_I, []),
}


class ObnError(RuntimeError):
    """A non-zero status from libobn, with the library's thread-local message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libobn error {code}: {message}")
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library first "
                "(python __graft_entry__.py build, or make -C 0xbitnet_b200/csrc)"
            )
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    m = lib().obn_error_message()
    return m.decode() if m else ""


def check(rc: int) -> None:
    if rc != OBN_OK:
        raise ObnError(rc, last_error())
