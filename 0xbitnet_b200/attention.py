"""Decode attention around the BitLinear path (host mirror over libobn's C ABI).

The reference's ``Attention::forward`` (packages/rust/crates/oxbitnet/src/nn/
attention.rs:85-124) projects q/k/v with BitLinear, applies RoPE (rope.wgsl),
appends k/v to an f32 KV cache, computes scores, softmax and the weighted sum
of V (attention.wgsl, softmax.wgsl), then the o projection. Here the q/k/v
projections are one merged BitLinear whose output feeds
``rope_kv_append`` (RoPE + an fp16 cache append in one kernel) and
``attention`` (split-KV GQA attention with a combine pass); the o projection
is a BitLinear again.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import check, lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class KVCache:
    """fp16 caches [B, S_max, Hkv, head_dim] for keys and values of one layer."""

    def __init__(self, B: int, S_max: int, Hkv: int, head_dim: int = 128, device=None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.k = torch.zeros((B, S_max, Hkv, head_dim), dtype=torch.float16, device=device)
        self.v = torch.zeros_like(self.k)
        self.B, self.S_max, self.Hkv, self.head_dim = B, S_max, Hkv, head_dim
        self.seq_len = 0


def rope_kv_append(qkv: torch.Tensor, cache: KVCache, H: int, n: int,
                   theta_base: float = 500000.0, q_out: torch.Tensor | None = None,
                   pos: int | None = None) -> torch.Tensor:
    """qkv [B*n, (H + 2*Hkv) * d] f32 of n new tokens per sequence -> rotated q
    [B*n, H*d]; k (rotated) and v stored at positions pos .. pos + n - 1
    (pos defaults to cache.seq_len)."""
    d = cache.head_dim
    q = q_out if q_out is not None else torch.empty((cache.B * n, H * d), dtype=torch.float32,
                                                     device=qkv.device)
    pos = cache.seq_len if pos is None else pos
    check(lib().obn_rope_kv_append(_ptr(qkv), cache.B, n, H, cache.Hkv, d, pos,
                                   ctypes.c_float(theta_base), _ptr(q), _ptr(cache.k),
                                   _ptr(cache.v), cache.S_max, _stream(qkv.device)))
    return q


def attention(q: torch.Tensor, cache: KVCache, H: int, n: int, seq_len: int,
              scale: float | None = None, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Causal GQA attention of the n newest tokens (the cache holds seq_len
    positions per sequence): q [B*n, H*d] -> out [B*n, H*d]."""
    d = cache.head_dim
    # attention.rs: scale = 1 / sqrt(head_dim) in f32
    sc = float(np.float32(1.0) / np.sqrt(np.float32(d))) if scale is None else scale
    out = out if out is not None else torch.empty_like(q)
    need = int(lib().obn_attention_workspace_bytes(cache.B, n, H, d, seq_len))
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    check(lib().obn_attention_decode(_ptr(q), _ptr(cache.k), _ptr(cache.v), cache.B, n, H,
                                     cache.Hkv, d, cache.S_max, seq_len, ctypes.c_float(sc),
                                     _ptr(out), _ptr(ws), ws.numel(), _stream(q.device)))
    return out


def attention_rope(qkv: torch.Tensor, cache: KVCache, H: int, pos: int,
                   theta_base: float = 500000.0, scale: float | None = None,
                   out: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One decode token per sequence: RoPE + KV append + attention in one pass
    (bit-identical to rope_kv_append then attention with n = 1). qkv [B,
    (H + 2*Hkv) * d] unrotated -> out [B, H*d]; the token sits at position pos."""
    d = cache.head_dim
    sc = float(np.float32(1.0) / np.sqrt(np.float32(d))) if scale is None else scale
    out = out if out is not None else torch.empty((cache.B, H * d), dtype=torch.float32,
                                                  device=qkv.device)
    need = int(lib().obn_attention_workspace_bytes(cache.B, 1, H, d, pos + 1))
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(max(need, 1), dtype=torch.uint8, device=qkv.device)
    check(lib().obn_attention_decode_rope(_ptr(qkv), _ptr(cache.k), _ptr(cache.v), cache.B, H,
                                          cache.Hkv, d, cache.S_max, pos,
                                          ctypes.c_float(theta_base), ctypes.c_float(sc),
                                          _ptr(out), _ptr(ws), ws.numel(), _stream(qkv.device)))
    cache.seq_len = max(cache.seq_len, pos + 1)
    return out
