"""Seeded synthetic Q/K/V in the reference's [B, H, N, d] bf16 layout.

The reference's generator draws U(-0.5, 0.5) (profile/gen_ref.py:54-56); the
benchmarked configurations use the distributions BASELINE.json names:
  "normal"   Q, K, V ~ N(0, 1)
  "peaked"   Q, K ~ N(0, std 3), V ~ U(-1, 1)   (stresses max-rescaling)
  "uniform"  Q, K, V ~ U(-0.5, 0.5)              (gen_ref.py's distribution)
Values are drawn in fp32 from a torch.Generator on `device` and cast to bf16.
"""
from __future__ import annotations

import torch

DISTS = ("normal", "peaked", "uniform")


def make_qkv(B: int, H: int, N: int, d: int = 64, dist: str = "normal", seed: int = 0,
             device: str | torch.device = "cpu"):
    if dist not in DISTS:
        raise ValueError(f"unknown distribution {dist!r}; expected one of {DISTS}")
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shape = (B, H, N, d)

    def normal(std: float):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)

    def uniform(lo: float, hi: float):
        return (torch.rand(shape, generator=g, device=device, dtype=torch.float32) * (hi - lo) + lo).to(torch.bfloat16)

    if dist == "normal":
        return normal(1.0), normal(1.0), normal(1.0)
    if dist == "peaked":
        return normal(3.0), normal(3.0), uniform(-1.0, 1.0)
    return uniform(-0.5, 0.5), uniform(-0.5, 0.5), uniform(-0.5, 0.5)
