"""The named workloads of the attention path and their seeded synthetic inputs.

Sequence order is text first, then image (the joint `cat([txt, img])` of
crates/foundry-spike/src/lib.rs:363-365). Axial positions (t, h, w, l):
text tokens at (0, 0, 0, 0), image token i of a G x G latent grid at
(0, i // G, i % G, 0). Inputs are drawn from one CPU torch.Generator in the
order q, k, v, dO with shape (B, S, H, D) in fp32, scaled, then cast.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class AttnConfig:
    name: str
    B: int
    H: int
    D: int
    txt: int
    grid: int
    dtype: torch.dtype
    qkv_scale: float
    seed: int = 0

    @property
    def S(self) -> int:
        return self.txt + self.grid * self.grid

    def flops_fwd(self) -> float:
        return 4.0 * self.B * self.H * self.S * self.S * self.D

    def flops_bwd(self) -> float:
        return 10.0 * self.B * self.H * self.S * self.S * self.D

    def flops_fwd_bwd(self) -> float:
        return 14.0 * self.B * self.H * self.S * self.S * self.D


CONFIGS = {
    # C1: CPU-runnable f32 case, 64 text + 16x16 image tokens
    "c1": AttnConfig("c1", B=1, H=8, D=128, txt=64, grid=16, dtype=torch.float32, qkv_scale=1.0),
    # C2: bf16, 512 text + 64x64 image tokens (a 1024^2 image at /16)
    "c2": AttnConfig("c2", B=1, H=24, D=128, txt=512, grid=64, dtype=torch.bfloat16, qkv_scale=0.5),
    # C4: batched training-step attention, B=8 of C2
    "c4": AttnConfig("c4", B=8, H=24, D=128, txt=512, grid=64, dtype=torch.bfloat16, qkv_scale=0.5),
    # C5: long sequence, 512 text + 128x128 image tokens (a 2048^2 image)
    "c5": AttnConfig("c5", B=1, H=24, D=128, txt=512, grid=128, dtype=torch.bfloat16, qkv_scale=0.5),
}


def positions(txt: int, grid: int) -> torch.Tensor:
    """(S, 4) fp32 axial positions, text then image."""
    n_img = grid * grid
    pos = torch.zeros((txt + n_img, 4), dtype=torch.float32)
    i = torch.arange(n_img)
    pos[txt:, 1] = (i // grid).float()
    pos[txt:, 2] = (i % grid).float()
    return pos


def make_inputs(cfg: AttnConfig, device="cpu", batch: int | None = None):
    """Seeded q, k, v, dO in the config's dtype on `device` (B, S, H, D)."""
    B = cfg.B if batch is None else batch
    g = torch.Generator().manual_seed(cfg.seed)
    shape = (B, cfg.S, cfg.H, cfg.D)
    q = torch.randn(shape, generator=g) * cfg.qkv_scale
    k = torch.randn(shape, generator=g) * cfg.qkv_scale
    v = torch.randn(shape, generator=g) * cfg.qkv_scale
    d_o = torch.randn(shape, generator=g)
    return tuple(t.to(cfg.dtype).to(device) for t in (q, k, v, d_o))
