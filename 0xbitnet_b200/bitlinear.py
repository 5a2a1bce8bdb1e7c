"""Host-side mirror of 0xBitNet's BitLinear interface over libobn's C ABI.

``BitLinear`` follows the reference's operator for this path:

* ``BitLinear(packed_weights, weight_scales, norm_weight, in_dim, out_dim)`` —
  ``BitLinear::new`` (packages/rust/crates/oxbitnet/src/nn/bitlinear.rs:31-49;
  TS constructor packages/core/src/nn/bitlinear.ts:47-66), over device buffers
  in the reference's layout (packed ``[out_dim, in_dim/16]`` u32 I2_S, per-row
  f32 scales, optional f32 RMSNorm gamma);
* ``BitLinear.from_i2s(tensor_bytes, in_dim, out_dim)`` — the GGUF loader's
  I2_S upload with per-tensor scale extraction
  (packages/rust/crates/oxbitnet/src/model/loader.rs:105-137);
* ``forward(input, n)`` — ``BitLinear::forward`` (bitlinear.rs:52-97;
  bitlinear.ts:117-169): ``[n, in_dim]`` f32 in, ``[n, out_dim]`` f32 out.

PyTorch is used only for device memory and the current CUDA stream; every
computation runs in libobn.so's sm_100a kernels.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import check, lib


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda_f32(t: torch.Tensor, name: str) -> None:
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32
            and t.is_contiguous()):
        raise TypeError(f"{name} must be a contiguous float32 CUDA tensor")


class BitLinear:
    """Ternary linear layer: RMSNorm -> absmax int8 quantize -> ternary matmul."""

    def __init__(self, packed_weights: torch.Tensor, weight_scales: torch.Tensor,
                 norm_weight: torch.Tensor | None, in_dim: int, out_dim: int,
                 eps: float = 1e-5):
        if not packed_weights.is_cuda or not weight_scales.is_cuda:
            raise TypeError("packed_weights and weight_scales must be CUDA tensors")
        if packed_weights.numel() * packed_weights.element_size() < out_dim * in_dim // 4:
            raise ValueError("packed_weights is smaller than out_dim * in_dim / 4 bytes")
        _require_cuda_f32(weight_scales, "weight_scales")
        if norm_weight is not None:
            _require_cuda_f32(norm_weight, "norm_weight")
        self.device = packed_weights.device
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().obn_bitlinear_create(
                _ptr(packed_weights), _ptr(weight_scales), _ptr(norm_weight),
                ctypes.c_float(eps), in_dim, out_dim, _stream(self.device),
                ctypes.byref(handle)))
        self._init(handle, in_dim, out_dim)

    @classmethod
    def from_i2s(cls, tensor: bytes | np.ndarray, in_dim: int, out_dim: int,
                 norm_weight: np.ndarray | None = None, eps: float = 1e-5,
                 device: int = 0) -> "BitLinear":
        """Loads one GGUF I2_S tensor (packed bytes + 32-byte scale trailer)."""
        buf = np.frombuffer(tensor, np.uint8) if isinstance(tensor, (bytes, bytearray)) \
            else np.ascontiguousarray(tensor, np.uint8).reshape(-1)
        nw = None if norm_weight is None else np.ascontiguousarray(norm_weight, np.float32)
        handle = ctypes.c_void_p()
        check(lib().obn_bitlinear_load_i2s(
            buf.ctypes.data_as(ctypes.c_void_p), buf.size, in_dim, out_dim,
            None if nw is None else nw.ctypes.data_as(ctypes.c_void_p),
            ctypes.c_float(eps), device, ctypes.byref(handle)))
        self = cls.__new__(cls)
        self.device = torch.device("cuda", device)
        self._init(handle, in_dim, out_dim)
        return self

    @classmethod
    def from_i2s_gated(cls, gate: bytes | np.ndarray, up: bytes | np.ndarray, in_dim: int,
                       out_dim: int, norm_weight: np.ndarray | None = None, eps: float = 1e-5,
                       device: int = 0) -> "BitLinear":
        """The gated FFN's gate and up projections (two GGUF I2_S tensors) as one
        layer whose forward is relu(x W_gate^T)^2 * (x W_up^T) (ffn.rs:70-79)."""
        bufs = [np.frombuffer(t, np.uint8) if isinstance(t, (bytes, bytearray))
                else np.ascontiguousarray(t, np.uint8).reshape(-1) for t in (gate, up)]
        nw = None if norm_weight is None else np.ascontiguousarray(norm_weight, np.float32)
        handle = ctypes.c_void_p()
        check(lib().obn_bitlinear_load_i2s_gated(
            bufs[0].ctypes.data_as(ctypes.c_void_p), bufs[0].size,
            bufs[1].ctypes.data_as(ctypes.c_void_p), bufs[1].size, in_dim, out_dim,
            None if nw is None else nw.ctypes.data_as(ctypes.c_void_p),
            ctypes.c_float(eps), device, ctypes.byref(handle)))
        self = cls.__new__(cls)
        self.device = torch.device("cuda", device)
        self._init(handle, in_dim, out_dim)
        return self

    @classmethod
    def create_gated(cls, gate_packed: torch.Tensor, gate_scales: torch.Tensor,
                     up_packed: torch.Tensor, up_scales: torch.Tensor,
                     norm_weight: torch.Tensor | None, in_dim: int, out_dim: int,
                     eps: float = 1e-5) -> "BitLinear":
        """from_i2s_gated over device tensors (I2_S rows [out_dim, in_dim/4] and
        row scales [out_dim] for gate and for up)."""
        for t, nm in ((gate_scales, "gate_scales"), (up_scales, "up_scales")):
            _require_cuda_f32(t, nm)
        if norm_weight is not None:
            _require_cuda_f32(norm_weight, "norm_weight")
        device = gate_packed.device
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(lib().obn_bitlinear_create_gated(
                _ptr(gate_packed), _ptr(gate_scales), _ptr(up_packed), _ptr(up_scales),
                _ptr(norm_weight), ctypes.c_float(eps), in_dim, out_dim, _stream(device),
                ctypes.byref(handle)))
        self = cls.__new__(cls)
        self.device = device
        self._init(handle, in_dim, out_dim)
        return self

    def _init(self, handle: ctypes.c_void_p, in_dim: int, out_dim: int) -> None:
        self._h = handle
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.rows = int(lib().obn_bitlinear_rows(handle))  # 2 * out_dim when gated
        self._ws: dict[int, torch.Tensor] = {}

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def set_activation(self, act: int) -> None:
        """A gated layer's activation of the gate: 0 = ReLU^2 (the default), 1 = SiLU
        (the "bitnet" architecture's FFN, ffn.rs:70-79)."""
        check(lib().obn_bitlinear_set_activation(self._h, act))

    def workspace_bytes(self, n: int) -> int:
        return int(lib().obn_bitlinear_workspace_bytes(self._h, n))

    def _workspace(self, n: int) -> torch.Tensor:
        need = self.workspace_bytes(n)
        ws = self._ws.get(self.device.index)
        if ws is None or ws.numel() < need:
            # torch's caching allocator returns 512-byte aligned blocks.
            ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
            self._ws[self.device.index] = ws
        return ws

    def forward(self, input: torch.Tensor, n: int | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """input [n, in_dim] f32 (CUDA) -> [n, out_dim] f32."""
        _require_cuda_f32(input, "input")
        if n is None:
            n = input.numel() // self.in_dim
        if input.numel() < n * self.in_dim:
            raise ValueError(f"input holds {input.numel()} values, need {n * self.in_dim}")
        if out is None:
            out = torch.empty((n, self.out_dim), dtype=torch.float32, device=self.device)
        ws = self._workspace(n)
        check(lib().obn_bitlinear_forward(self._h, _ptr(input), n, _ptr(out), _ptr(ws),
                                          ws.numel(), _stream(self.device)))
        return out

    __call__ = forward

    def forward_residual(self, input: torch.Tensor, y: torch.Tensor,
                         n: int | None = None) -> torch.Tensor:
        """y += forward(input) in the matmul epilogue (the residual add after
        o_proj / down_proj, transformer.rs:63,69); y [n, out_dim] f32."""
        _require_cuda_f32(input, "input")
        _require_cuda_f32(y, "y")
        if n is None:
            n = input.numel() // self.in_dim
        ws = self._workspace(n)
        check(lib().obn_bitlinear_forward_residual(self._h, _ptr(input), n, _ptr(y), _ptr(ws),
                                                   ws.numel(), _stream(self.device)))
        return y

    def forward_tp(self, input: torch.Tensor, out_total: int, col0: int,
                   out_mc: int | None = None, out_ranks: list[int] | None = None,
                   n: int | None = None) -> None:
        """Tensor-parallel forward: this layer holds rows [col0, col0 + out_dim) of
        an out_total-row weight; writes them into columns [col0, col0 + out_dim) of
        every rank's [n, out_total] f32 output, through the multicast address
        `out_mc` or the per-rank device addresses `out_ranks` (ints). The caller
        orders all ranks' calls before reading (a barrier on the stream)."""
        _require_cuda_f32(input, "input")
        if n is None:
            n = input.numel() // self.in_dim
        if (out_mc is None) == (out_ranks is None):
            raise ValueError("give exactly one of out_mc and out_ranks")
        world = len(out_ranks) if out_ranks is not None else self._tp_world
        ranks = None
        if out_ranks is not None:
            ranks = (ctypes.c_void_p * len(out_ranks))(*[ctypes.c_void_p(p) for p in out_ranks])
        ws = self._workspace(n)
        check(lib().obn_bitlinear_forward_tp(
            self._h, _ptr(input), n, ctypes.c_void_p(out_mc) if out_mc is not None else None,
            ranks, world, out_total, col0, _ptr(ws), ws.numel(), _stream(self.device)))

    _tp_world = 1

    def matmul(self, q: torch.Tensor, scales: torch.Tensor, qsum: torch.Tensor,
               n: int | None = None) -> torch.Tensor:
        """Ternary GEMV/GEMM on already-quantized activations (int8 [n, in_dim])."""
        n = q.shape[0] if n is None else n
        out = torch.empty((n, self.rows), dtype=torch.float32, device=self.device)
        check(lib().obn_ternary_matmul(self._h, _ptr(q), _ptr(scales), _ptr(qsum), n,
                                       _ptr(out), _stream(self.device)))
        return out

    def acc(self, q: torch.Tensor, qsum: torch.Tensor) -> torch.Tensor:
        """Exact int32 accumulators sum_k w[m,k] q[t,k] -> [n, out_dim]."""
        n = q.shape[0]
        out = torch.empty((n, self.rows), dtype=torch.int32, device=self.device)
        check(lib().obn_ternary_acc(self._h, _ptr(q), _ptr(qsum), n, _ptr(out),
                                    _stream(self.device)))
        return out

    def export_i2s(self) -> torch.Tensor:
        """Device weights back in I2_S rows [out_dim, in_dim/4] (uint8)."""
        out = torch.empty((self.rows, self.in_dim // 4), dtype=torch.uint8, device=self.device)
        check(lib().obn_bitlinear_export_i2s(self._h, _ptr(out), _stream(self.device)))
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().obn_bitlinear_free(self._h)
            self._h = None
            self._ws.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def rmsnorm_quantize(x: torch.Tensor, norm_weight: torch.Tensor | None = None,
                     eps: float = 1e-5):
    """Fused rmsnorm.wgsl + quantize.wgsl -> (q int8 [n, d], scales f32 [n], qsum i32 [n])."""
    _require_cuda_f32(x, "x")
    if norm_weight is not None:
        _require_cuda_f32(norm_weight, "norm_weight")
    n, d = x.reshape(-1, x.shape[-1]).shape
    q = torch.empty((n, d), dtype=torch.int8, device=x.device)
    s = torch.empty(n, dtype=torch.float32, device=x.device)
    qs = torch.empty(n, dtype=torch.int32, device=x.device)
    check(lib().obn_rmsnorm_quantize(_ptr(x), _ptr(norm_weight), ctypes.c_float(eps), n, d,
                                     _ptr(q), _ptr(s), _ptr(qs), _stream(x.device)))
    return q, s, qs


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """rmsnorm.wgsl: (x * rsqrt(mean(x^2) + eps)) * weight."""
    _require_cuda_f32(x, "x")
    _require_cuda_f32(weight, "weight")
    n, d = x.reshape(-1, x.shape[-1]).shape
    y = torch.empty_like(x)
    check(lib().obn_rmsnorm(_ptr(x), _ptr(weight), ctypes.c_float(eps), n, d, _ptr(y),
                            _stream(x.device)))
    return y


def lm_head_f16(embed: torch.Tensor, x: torch.Tensor, norm_weight: torch.Tensor | None = None,
                eps: float = 1e-5) -> torch.Tensor:
    """The f16 LM head behind the final RMSNorm (model.rs:226-262; f32_matmul.wgsl):
    embed [vocab, dim] float16 and x [n, dim] f32 on one CUDA device ->
    logits [n, vocab] f32."""
    if not (embed.is_cuda and embed.dtype == torch.float16 and embed.is_contiguous()):
        raise TypeError("embed must be a contiguous float16 CUDA tensor")
    _require_cuda_f32(x, "x")
    if norm_weight is not None:
        _require_cuda_f32(norm_weight, "norm_weight")
    vocab, dim = embed.shape
    n = x.numel() // dim
    logits = torch.empty((n, vocab), dtype=torch.float32, device=x.device)
    check(lib().obn_lm_head_f16(_ptr(embed), vocab, dim, _ptr(x), _ptr(norm_weight),
                                ctypes.c_float(eps), n, _ptr(logits), _stream(x.device)))
    return logits


def lm_head_f16_batched(embed: torch.Tensor, x: torch.Tensor,
                        norm_weight: torch.Tensor | None = None, eps: float = 1e-5,
                        out: torch.Tensor | None = None,
                        workspace: torch.Tensor | None = None) -> torch.Tensor:
    """lm_head_f16 for many tokens on the tensor cores (hi/lo f16 split)."""
    if not (embed.is_cuda and embed.dtype == torch.float16 and embed.is_contiguous()):
        raise TypeError("embed must be a contiguous float16 CUDA tensor")
    _require_cuda_f32(x, "x")
    vocab, dim = embed.shape
    n = x.numel() // dim
    logits = out if out is not None else torch.empty((n, vocab), dtype=torch.float32,
                                                     device=x.device)
    need = int(lib().obn_lm_head_workspace_bytes(n, dim))
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib().obn_lm_head_f16_batched(_ptr(embed), vocab, dim, _ptr(x), _ptr(norm_weight),
                                        ctypes.c_float(eps), n, _ptr(logits), _ptr(ws),
                                        ws.numel(), _stream(x.device)))
    return logits


def check_device_errors() -> None:
    """Raises ObnError if a bounded in-kernel wait gave up since the last check."""
    check(lib().obn_check_device_errors())


__all__ = ["BitLinear", "rmsnorm_quantize", "rmsnorm", "check_device_errors", "_lib"]
