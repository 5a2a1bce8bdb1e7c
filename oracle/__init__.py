"""CPU oracle for 0xBitNet's ternary BitLinear path — TEST INFRASTRUCTURE ONLY.

ctypes wrapper over ``oracle/_build/libobn_oracle.so`` (built from
``oracle/obn_oracle.c`` by ``oracle/Makefile``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
import this module, and only as the checker. The shipped library under
``0xbitnet_b200/`` never imports it.

Each wrapper names the reference shader or helper it restates; the C source
carries the file:line citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libobn_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build() -> str:
    """Compile the oracle with its Makefile (system gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
            os.path.join(_HERE, "obn_oracle.c")
        ):
            build()
        L = ctypes.CDLL(_SO)
        L.orc_mulberry32_next.restype = ctypes.c_double
        L.orc_i2s_pack_row.restype = ctypes.c_size_t
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_half_to_float.restype = ctypes.c_float
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


# ---- seeded generators (tensor-utils.ts:9-48) -------------------------------
def randf32(n: int, seed: int = 42) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_randf32(_p(out, _f32p), ctypes.c_size_t(n), ctypes.c_uint32(seed & 0xFFFFFFFF))
    return out


def rand_ternary(n: int, seed: int = 42) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_rand_ternary(_p(out, _i8p), ctypes.c_size_t(n), ctypes.c_uint32(seed & 0xFFFFFFFF))
    return out


def rand_int8(n: int, seed: int = 42) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().orc_rand_int8(_p(out, _i32p), ctypes.c_size_t(n), ctypes.c_uint32(seed & 0xFFFFFFFF))
    return out


# ---- I2_S (i2s-pack.ts) -----------------------------------------------------
def i2s_pack_row(values: np.ndarray, K: int) -> np.ndarray:
    v = np.ascontiguousarray(values, np.int8)
    out = np.zeros(((K + 127) // 128) * 32, np.uint8)
    lib().orc_i2s_pack_row(_p(v, _i8p), ctypes.c_int(K), _p(out, _u8p))
    return out


def i2s_unpack_row(packed: np.ndarray, K: int) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.uint8)
    out = np.empty(K, np.int8)
    lib().orc_i2s_unpack_row(_p(p, _u8p), ctypes.c_int(K), _p(out, _i8p))
    return out


def i2s_pack_matrix(values: np.ndarray) -> np.ndarray:
    """[M, K] ternary (K % 128 == 0) -> [M, K/4] uint8 I2_S rows."""
    v = np.ascontiguousarray(values, np.int8)
    M, K = v.shape
    assert K % 128 == 0
    out = np.empty((M, K // 4), np.uint8)
    lib().orc_i2s_pack_matrix(_p(v, _i8p), ctypes.c_int(M), ctypes.c_int(K), _p(out, _u8p))
    return out


def i2s_unpack_matrix(packed: np.ndarray, K: int) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.uint8)
    return np.stack([i2s_unpack_row(p[m], K) for m in range(p.shape[0])])


# ---- kernels ------------------------------------------------------------------
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """rmsnorm.wgsl:40-62."""
    x = np.ascontiguousarray(x, np.float32)
    N, D = x.reshape(-1, x.shape[-1]).shape
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x, _f32p), _p(w, _f32p), N, D, ctypes.c_float(eps), _p(y, _f32p))
    return y


def quantize(x: np.ndarray):
    """quantize.wgsl:41-73 -> (q int8 [N, D], scales f32 [N])."""
    x = np.ascontiguousarray(x, np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    N, D = x2.shape
    q = np.empty((N, D), np.int8)
    s = np.empty(N, np.float32)
    lib().orc_quantize(_p(x2, _f32p), N, D, _p(q, _i8p), _p(s, _f32p))
    return q, s


def ternary_acc(w_i2s: np.ndarray, q: np.ndarray, M: int, K: int) -> np.ndarray:
    """int32 accumulators acc[n, m] = sum_k t[m, k] q[n, k]."""
    w = np.ascontiguousarray(w_i2s, np.uint8)
    q2 = np.ascontiguousarray(q, np.int8).reshape(-1, K)
    N = q2.shape[0]
    acc = np.empty((N, M), np.int32)
    lib().orc_ternary_acc(_p(w, _u8p), _p(q2, _i8p), M, N, K, _p(acc, _i32p))
    return acc


def ternary_acc_omp(w_i2s: np.ndarray, q: np.ndarray, M: int, K: int,
                    threads: int = 0) -> np.ndarray:
    """ternary_acc with rows split over OpenMP threads (identical results; for the
    large test shapes)."""
    w = np.ascontiguousarray(w_i2s, np.uint8)
    q2 = np.ascontiguousarray(q, np.int8).reshape(-1, K)
    N = q2.shape[0]
    acc = np.empty((N, M), np.int32)
    lib().orc_ternary_acc_omp(_p(w, _u8p), _p(q2, _i8p), M, N, K, _p(acc, _i32p),
                              ctypes.c_int(threads))
    return acc


def ternary_gemv(w_i2s, q, s_w, s_x: float, M: int, K: int) -> np.ndarray:
    """ternary_gemv.wgsl:55-96."""
    w = np.ascontiguousarray(w_i2s, np.uint8)
    q1 = np.ascontiguousarray(q, np.int8).reshape(K)
    sw = np.ascontiguousarray(s_w, np.float32)
    out = np.empty(M, np.float32)
    lib().orc_ternary_gemv(_p(w, _u8p), _p(q1, _i8p), _p(sw, _f32p), ctypes.c_float(s_x), M, K,
                           _p(out, _f32p))
    return out


def ternary_gemm(w_i2s, q, s_w, s_x, M: int, K: int) -> np.ndarray:
    """ternary_gemm.wgsl:56-135 -> [N, M]."""
    w = np.ascontiguousarray(w_i2s, np.uint8)
    q2 = np.ascontiguousarray(q, np.int8).reshape(-1, K)
    N = q2.shape[0]
    sw = np.ascontiguousarray(s_w, np.float32)
    sx = np.ascontiguousarray(s_x, np.float32)
    out = np.empty((N, M), np.float32)
    lib().orc_ternary_gemm(_p(w, _u8p), _p(q2, _i8p), _p(sw, _f32p), _p(sx, _f32p), M, N, K,
                           _p(out, _f32p))
    return out


def bitlinear(x, w_i2s, s_w, M: int, K: int, norm_w=None, eps: float = 1e-5):
    """bitlinear.rs:52-97 -> (out [n, M], q [n, K], scales [n])."""
    x2 = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    n = x2.shape[0]
    w = np.ascontiguousarray(w_i2s, np.uint8)
    sw = np.ascontiguousarray(s_w, np.float32)
    nw = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
    out = np.empty((n, M), np.float32)
    q = np.empty((n, K), np.int8)
    s = np.empty(n, np.float32)
    lib().orc_bitlinear(_p(x2, _f32p), n, None if nw is None else _p(nw, _f32p),
                        ctypes.c_float(eps), _p(w, _u8p), _p(sw, _f32p), M, K, _p(out, _f32p),
                        _p(q, _i8p), _p(s, _f32p))
    return out, q, s


def bitlinear_omp(x, w_i2s, s_w, M: int, K: int, norm_w=None, eps: float = 1e-5,
                  threads: int = 0) -> np.ndarray:
    """Row-parallel bitlinear (identical results) for the timed CPU baseline."""
    x2 = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    n = x2.shape[0]
    w = np.ascontiguousarray(w_i2s, np.uint8)
    sw = np.ascontiguousarray(s_w, np.float32)
    nw = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
    out = np.empty((n, M), np.float32)
    lib().orc_bitlinear_omp(_p(x2, _f32p), n, None if nw is None else _p(nw, _f32p),
                            ctypes.c_float(eps), _p(w, _u8p), _p(sw, _f32p), M, K,
                            _p(out, _f32p), ctypes.c_int(threads))
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ---- LM head (f32_matmul.wgsl:27-74; final RMSNorm: rmsnorm.wgsl) ----------
def half_to_float(bits: int) -> float:
    """binary16 bit pattern -> float32 (unpack2x16float), one value."""
    return float(lib().orc_half_to_float(bits & 0xFFFF))


def lm_head_f16(hidden: np.ndarray, embed: np.ndarray, norm_w: np.ndarray | None = None,
                eps: float = 1e-5) -> np.ndarray:
    """logits [N, V] = RMSNorm(hidden) (when norm_w is given) times the f16
    embedding [V, D], in the shader's per-lane order and halving tree."""
    h = np.ascontiguousarray(hidden, np.float32)
    D = h.shape[-1]
    h = h.reshape(-1, D)
    if norm_w is not None:
        h = rmsnorm(h, norm_w, eps)
    e = np.ascontiguousarray(embed, np.float16).view(np.uint16)
    V = e.shape[0]
    out = np.empty((h.shape[0], V), np.float32)
    lib().orc_lm_head_f16(_p(h, _f32p), _p(e, _u16p), h.shape[0], V, D, _p(out, _f32p))
    return out


def f32_matmul_seq(hidden: np.ndarray, embed: np.ndarray, N: int, V: int, D: int) -> np.ndarray:
    """reference.ts:342-360 refF32Matmul: sequential f32 sum per (n, v)."""
    h = np.ascontiguousarray(hidden, np.float32)
    e = np.ascontiguousarray(embed, np.float32)
    out = np.empty(N * V, np.float32)
    lib().orc_f32_matmul_seq(_p(h, _f32p), _p(e, _f32p), N, V, D, _p(out, _f32p))
    return out


# ---- gated FFN (ffn.rs:70-79: activation.wgsl ReLU^2, elementwise.wgsl multiply)
def relu2_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, np.float32)
    u = np.ascontiguousarray(up, np.float32)
    y = np.empty_like(g)
    lib().orc_relu2_mul(_p(g, _f32p), _p(u, _f32p), ctypes.c_size_t(g.size), _p(y, _f32p))
    return y


# ---- attention (rope.wgsl, attention.wgsl, softmax.wgsl; attention.rs:85-124)
def rope(x: np.ndarray, heads: int, head_dim: int, pos_offset: int,
         theta_base: float = 500000.0) -> np.ndarray:
    """x [N, heads*head_dim] -> rotated copy (rope.wgsl:27-56)."""
    y = np.ascontiguousarray(x, np.float32).copy()
    N = y.size // (heads * head_dim)
    lib().orc_rope(_p(y, _f32p), N, heads, head_dim, pos_offset, ctypes.c_float(theta_base))
    return y


def attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, H: int, Hkv: int, d: int,
              scale: float | None = None) -> np.ndarray:
    """One sequence: q [N, H*d], K/V [S, Hkv*d] (S includes the N new tokens,
    causal) -> out [N, H*d]."""
    q = np.ascontiguousarray(q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    N = q.size // (H * d)
    S = K.size // (Hkv * d)
    sc = float(np.float32(1.0) / np.sqrt(np.float32(d))) if scale is None else scale
    out = np.empty((N, H * d), np.float32)
    lib().orc_attention(_p(q, _f32p), _p(K, _f32p), _p(V, _f32p), N, S, H, Hkv, d,
                        ctypes.c_float(sc), _p(out, _f32p))
    return out
