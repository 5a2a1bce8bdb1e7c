"""A BitNet b1.58 decoder step on libobn's kernels (config 3: decode tok/s).

Mirrors the reference's forward (packages/rust/crates/oxbitnet/src/nn/
model.rs:200-262 and transformer.rs:51-72) for one new token per sequence:

    x = embed(ids)                                        embedding.wgsl
    per layer:
      qkv = BitLinear_qkv(RMSNorm(x; input_layernorm))    q/k/v projections on
                                                          one normed input
      q = RoPE(q); k, v -> fp16 KV cache; a = attention   attention.rs:85-124
      x = x + BitLinear_o(a; attn_sub_norm)               dispatch_add
      g = relu(gate)^2 * up of RMSNorm(x; post_attn)      ffn.rs:70-79
      x = x + BitLinear_down(g; ffn_sub_norm)
    logits = LM head (tied f16 embedding) of RMSNorm(x; final norm)

B200 form: the block RMSNorms are the fused RMSNorm of the BitLinear that
consumes them (numerically the same: rmsnorm then quantize), the residual adds
happen in the o_proj / down_proj epilogues (x + y rounded once, as the add
kernel would), q/k/v are one
merged 3840-row BitLinear with a per-row scale table, gate and up are one
interleaved gated layer, and the KV cache is fp16; small batches rotate q and
append k/v inside the attention pass (one launch fewer). Every step is a fixed
sequence of libobn launches on one stream, so it is captured as a CUDA graph.
Two or more sequences take the tensor-core LM head (f16 hi/lo split, f32
accumulation) instead of the shader-order one. Weights are random (seeded)
with the reference's distributions; no checkpoint is needed to measure speed.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import attention as att
from ._lib import check, lib
from .bitlinear import BitLinear, lm_head_f16, lm_head_f16_batched, rmsnorm
from .diagnose import stage_stats


# Batches up to this size take the fused RoPE + attention pass (one launch fewer);
# larger ones rotate q once in a separate pass instead of once per KV chunk.
FUSED_ROPE_MAX_BATCH = 8


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


@dataclass
class DecoderConfig:
    layers: int = 30
    hidden: int = 2560
    ffn: int = 6912
    heads: int = 20
    kv_heads: int = 5
    head_dim: int = 128
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5


def _ternary_rows(g: torch.Generator, M: int, K: int, device) -> torch.Tensor:
    """I2_S rows [M, K/4] of i.i.d. ternary weights, P(-1)=P(+1)=0.3."""
    u = torch.rand((M, K), generator=g, device=device)
    codes = torch.where(u < 0.3, 0, torch.where(u < 0.7, 1, 2)).to(torch.uint8)
    del u
    c = codes.view(M, K // 128, 4, 32)
    return ((c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]).reshape(
        M, K // 4).contiguous()


def _scale(g: torch.Generator, device) -> float:
    return float(0.5 + 1.5 * torch.rand((), generator=g, device=device).item())


def _gamma(g: torch.Generator, K: int, device) -> torch.Tensor:
    return (1.0 + 0.1 * torch.randn((K,), generator=g, device=device)).float()


class DecoderLayer:
    """One transformer block's weights on the device, as libobn layers. With
    keep_source, the generated I2_S rows are also kept on the host (`source`:
    name -> uint8 [rows, in/4]) as they were before the device repack, so a
    checker can rebuild the block from them."""

    def __init__(self, cfg: DecoderConfig, g: torch.Generator, device,
                 keep_source: bool = False):
        D, F, H, Hkv, d = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
        nq, nk = H * d, Hkv * d
        self.source = {} if keep_source else None
        # q, k, v: three ternary tensors with their own scales -> one layer
        rows = [_ternary_rows(g, m, D, device) for m in (nq, nk, nk)]
        if keep_source:
            self.source["qkv"] = torch.cat(rows).cpu().numpy()
        scales = [_scale(g, device) for _ in range(3)]
        self.qkv_scales = scales  # per-tensor scales of q, k, v (kept for checks)
        s_w = torch.cat([torch.full((m,), s, dtype=torch.float32, device=device)
                         for m, s in zip((nq, nk, nk), scales)])
        self.attn_norm = _gamma(g, D, device)
        self.qkv = BitLinear(torch.cat(rows), s_w, self.attn_norm, D, nq + 2 * nk, cfg.eps)
        del rows
        self.attn_sub_norm = _gamma(g, nq, device)
        o = _ternary_rows(g, D, nq, device)
        if keep_source:
            self.source["o"] = o.cpu().numpy()
        self.o_scale = _scale(g, device)
        self.o = BitLinear(o, torch.full((D,), self.o_scale, device=device),
                           self.attn_sub_norm, nq, D, cfg.eps)
        self.ffn_norm = _gamma(g, D, device)
        gate, up = _ternary_rows(g, F, D, device), _ternary_rows(g, F, D, device)
        if keep_source:
            self.source["gate"], self.source["up"] = gate.cpu().numpy(), up.cpu().numpy()
        self.gate_scale, self.up_scale = _scale(g, device), _scale(g, device)
        self.gate_up = BitLinear.create_gated(
            gate, torch.full((F,), self.gate_scale, device=device),
            up, torch.full((F,), self.up_scale, device=device), self.ffn_norm, D, F, cfg.eps)
        del gate, up
        self.ffn_sub_norm = _gamma(g, F, device)
        dn = _ternary_rows(g, D, F, device)
        if keep_source:
            self.source["down"] = dn.cpu().numpy()
        self.down_scale = _scale(g, device)
        self.down = BitLinear(dn, torch.full((D,), self.down_scale, device=device),
                              self.ffn_sub_norm, F, D, cfg.eps)

    def close(self):
        for L in (self.qkv, self.o, self.gate_up, self.down):
            L.close()


class BitNetDecoder:
    """B sequences decoding one token per step, KV caches of `ctx` positions."""

    def __init__(self, cfg: DecoderConfig, B: int, ctx: int, device=None, seed: int = 0,
                 keep_source: bool = False):
        self.cfg, self.B, self.ctx = cfg, B, ctx
        self.device = device if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        dev = self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        with torch.cuda.device(dev):
            self.layers = [DecoderLayer(cfg, g, dev, keep_source) for _ in range(cfg.layers)]
            self.embed = (0.02 * torch.randn((cfg.vocab, cfg.hidden), generator=g,
                                             device=dev)).to(torch.float16)
            self.final_norm = _gamma(g, cfg.hidden, dev)
            self.caches = [att.KVCache(B, ctx, cfg.kv_heads, cfg.head_dim, device=dev)
                           for _ in range(cfg.layers)]
            D, H, d = cfg.hidden, cfg.heads, cfg.head_dim
            f32 = dict(dtype=torch.float32, device=dev)
            self.x = torch.empty((B, D), **f32)
            self.qkv_out = torch.empty((B, (H + 2 * cfg.kv_heads) * d), **f32)
            self.q = torch.empty((B, H * d), **f32)
            self.attn = torch.empty((B, H * d), **f32)
            self.o_out = torch.empty((B, D), **f32)
            self.ffn_out = torch.empty((B, cfg.ffn), **f32)
            self.down_out = torch.empty((B, D), **f32)
            self.ids = torch.zeros((B,), dtype=torch.int32, device=dev)
            self.attn_ws = torch.empty(max(1, int(lib().obn_attention_workspace_bytes(
                B, 1, H, d, ctx))), dtype=torch.uint8, device=dev)
            self.logits = torch.empty((B, cfg.vocab), **f32)
            self.lm_ws = torch.empty(max(1, int(lib().obn_lm_head_workspace_bytes(B, D))),
                                     dtype=torch.uint8, device=dev)

    def fill_caches(self, seq_len: int, seed: int = 1) -> None:
        """Stands in for a prefill: random fp16 keys/values at positions < seq_len."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for c in self.caches:
            c.k[:, :seq_len].normal_(generator=g)
            c.v[:, :seq_len].normal_(generator=g)
            c.seq_len = seq_len

    def _embed(self, s) -> None:
        cfg = self.cfg
        check(lib().obn_embed_f16(_ptr(self.embed), cfg.vocab, cfg.hidden, _ptr(self.ids),
                                  self.B, _ptr(self.x), s))

    def _layer(self, L, c, pos: int) -> None:
        """One transformer block on self.x in place (transformer.rs:51-72)."""
        cfg, B, H = self.cfg, self.B, self.cfg.heads
        L.qkv.forward(self.x, n=B, out=self.qkv_out)
        if B <= FUSED_ROPE_MAX_BATCH:  # RoPE + KV append + attention in one pass
            att.attention_rope(self.qkv_out, c, H, pos, cfg.rope_theta, out=self.attn,
                               workspace=self.attn_ws)
        else:  # every split CTA would rotate its q heads again: rotate once first
            att.rope_kv_append(self.qkv_out, c, H, 1, cfg.rope_theta, q_out=self.q, pos=pos)
            att.attention(self.q, c, H, 1, pos + 1, out=self.attn, workspace=self.attn_ws)
        L.o.forward_residual(self.attn, self.x, n=B)  # x += o_proj(attn)
        L.gate_up.forward(self.x, n=B, out=self.ffn_out)
        L.down.forward_residual(self.ffn_out, self.x, n=B)  # x += down(ffn)

    def _lm_head(self) -> torch.Tensor:
        cfg = self.cfg
        if self.B == 1:  # the shader's exact order (the reference's own case is one token)
            return lm_head_f16(self.embed, self.x, self.final_norm, cfg.eps)
        # two or more tokens: the tensor-core head reads the table once for all of
        # them (the exact-order kernel is bound by its unfused f32 products there)
        return lm_head_f16_batched(self.embed, self.x, self.final_norm, cfg.eps,
                                   out=self.logits, workspace=self.lm_ws)

    def step(self, pos: int) -> torch.Tensor:
        """Enqueues one decode step for the tokens in self.ids at position `pos`
        (every cache holds pos positions before it); returns logits [B, vocab]."""
        self._embed(_stream(self.device))
        for L, c in zip(self.layers, self.caches):
            self._layer(L, c, pos)
        return self._lm_head()

    def diagnose(self, pos: int) -> list[dict]:
        """The decode step of `step(pos)`, stage by stage, with the reference's
        diagnostic statistics of each stage (model.ts:449-531): the embedding, the
        hidden state after layers 0 and 1 and after the last layer, the final
        RMSNorm, the LM-head input (every sequence's row: one token each) and the
        first 100 logits of sequence 0. Synchronises after every stage; the caches
        take the step's k / v as `step` would."""
        cfg = self.cfg
        host = lambda t: t.detach().float().cpu().numpy()
        out = []
        self._embed(_stream(self.device))
        out.append(stage_stats("embedding", host(self.x)))
        for i, (L, c) in enumerate(zip(self.layers, self.caches)):
            self._layer(L, c, pos)
            if i < 2:
                out.append(stage_stats(f"layer_{i}", host(self.x)))
        out.append(stage_stats("last_layer", host(self.x)))
        normed = host(rmsnorm(self.x, self.final_norm, cfg.eps))
        out.append(stage_stats("final_norm", normed))
        out.append(stage_stats("lm_input", normed))
        logits = self._lm_head()
        out.append(stage_stats("logits_first100", host(logits[0, :100])))
        return out

    def close(self) -> None:
        for L in self.layers:
            L.close()
