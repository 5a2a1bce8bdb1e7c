"""Host-side I2_S helpers: build and split GGUF I2_S tensors (numpy, vectorised).

Layout (packages/core/src/shaders/__tests__/helpers/i2s-pack.ts:30-58 and
packages/rust/crates/oxbitnet/src/model/loader.rs:105-137): each output row is
in_dim/4 bytes of 128-element blocks; byte gp of a block holds the 2-bit codes
(weight + 1) of elements gp, 32+gp, 64+gp, 96+gp in bits 7:6, 5:4, 3:2, 1:0.
A GGUF I2_S tensor is the packed rows followed by 32 bytes whose first float32
is the per-tensor weight scale (the reference replicates it 8 times).
"""
from __future__ import annotations

import numpy as np

BLOCK = 128


def pack_rows(values: np.ndarray) -> np.ndarray:
    """Ternary [M, K] (K % 128 == 0) -> I2_S rows [M, K/4] uint8."""
    v = np.asarray(values)
    M, K = v.shape
    if K % BLOCK:
        raise ValueError(f"K={K} is not a multiple of {BLOCK}")
    codes = (v.astype(np.int16) + 1).astype(np.uint8).reshape(M, K // BLOCK, 4, 32)
    packed = (codes[:, :, 0] << 6) | (codes[:, :, 1] << 4) | (codes[:, :, 2] << 2) | codes[:, :, 3]
    return packed.reshape(M, K // 4)


def unpack_rows(packed: np.ndarray, K: int) -> np.ndarray:
    """I2_S rows [M, K/4] -> ternary int8 [M, K]."""
    p = np.asarray(packed, np.uint8).reshape(-1, K // BLOCK, 32)
    g = np.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], axis=2)
    return (g.astype(np.int8) - 1).reshape(p.shape[0], K)


def make_tensor(packed_rows: np.ndarray, scale: float) -> np.ndarray:
    """Packed rows + 32-byte trailer (scale replicated 8x) -> one GGUF I2_S blob."""
    trailer = np.full(8, scale, dtype="<f4").view(np.uint8)
    return np.concatenate([np.ascontiguousarray(packed_rows, np.uint8).reshape(-1), trailer])


def split_tensor(blob: np.ndarray, in_dim: int, out_dim: int):
    """GGUF I2_S blob -> (packed rows [out_dim, in_dim/4], scale)."""
    b = np.asarray(blob, np.uint8).reshape(-1)
    n = out_dim * in_dim // 4
    if b.size < n + 32:
        raise ValueError(f"I2_S tensor needs {n + 32} bytes, got {b.size}")
    return b[:n].reshape(out_dim, in_dim // 4), float(b[n:n + 4].view("<f4")[0])


def random_ternary(rng: np.random.Generator, M: int, K: int,
                   p_neg: float = 0.3, p_zero: float = 0.4) -> np.ndarray:
    """i.i.d. ternary weights with P(-1)=p_neg, P(0)=p_zero, P(+1)=rest."""
    u = rng.random((M, K), dtype=np.float32)
    return np.where(u < p_neg, -1, np.where(u < p_neg + p_zero, 0, 1)).astype(np.int8)
