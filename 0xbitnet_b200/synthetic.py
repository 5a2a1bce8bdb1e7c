"""Seeded synthetic BitLinear workloads with the benchmark's shapes and distributions.

The reference publishes no benchmark dataset for this path; its configs name
synthetic inputs (activations ~N(0,1), RMSNorm gamma ~N(1, 0.1), eps 1e-5,
i.i.d. ternary weights with P(-1)=P(+1)=0.3, P(0)=0.4, one per-tensor scale
~U(0.5, 2)). Every generator here is deterministic in its seed (numpy
default_rng), so tests, fixtures and benchmarks see identical data.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import i2s

# BitNet-b1.58-2B layer shapes (out x in): fused QKV, o_proj, gate, up, down.
SHAPES_2B = {
    "qkv": (3840, 2560),
    "o": (2560, 2560),
    "gate": (6912, 2560),
    "up": (6912, 2560),
    "down": (2560, 6912),
}
# 3B-class prefill shapes (hidden 3072, FFN 9216; QKV assumed MHA).
SHAPES_3B = {
    "qkv": (9216, 3072),
    "o": (3072, 3072),
    "gate": (9216, 3072),
    "up": (9216, 3072),
    "down": (3072, 9216),
}


@dataclass
class LayerData:
    packed: np.ndarray     # I2_S rows [M, K/4] uint8
    scale: float           # per-tensor weight scale
    gamma: np.ndarray      # RMSNorm weight [K] f32
    M: int
    K: int

    def blob(self) -> np.ndarray:
        return i2s.make_tensor(self.packed, self.scale)

    def row_scales(self) -> np.ndarray:
        return np.full(self.M, self.scale, np.float32)


def layer(seed: int, M: int, K: int) -> LayerData:
    rng = np.random.default_rng(seed)
    w = i2s.random_ternary(rng, M, K)
    scale = float(np.float32(rng.uniform(0.5, 2.0)))
    gamma = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    return LayerData(i2s.pack_rows(w), scale, gamma, M, K)


def activations(seed: int, n: int, K: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((n, K)).astype(np.float32)


def layer_device(seed: int, M: int, K: int, device="cuda"):
    """Same distributions as layer(), generated on the GPU (fast for large stacks).

    Returns (packed [M, K/4] uint8 I2_S rows, row scales [M] f32, gamma [K] f32)
    as CUDA tensors. The values differ from layer(seed) (different generator).
    """
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    u = torch.rand((M, K), generator=g, device=device)
    codes = torch.where(u < 0.3, 0, torch.where(u < 0.7, 1, 2)).to(torch.uint8)
    del u
    c = codes.view(M, K // 128, 4, 32)
    packed = ((c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3])
    packed = packed.reshape(M, K // 4).contiguous()
    scale = float(0.5 + 1.5 * torch.rand((), generator=g, device=device).item())
    s_w = torch.full((M,), scale, dtype=torch.float32, device=device)
    gamma = (1.0 + 0.1 * torch.randn((K,), generator=g, device=device)).float()
    return packed, s_w, gamma
