"""Test support for the block callers (`foundry_trainer_b200.blocks`).

TEST INFRASTRUCTURE ONLY.

`TorchJointAttention` / `TorchSingleAttention` have the call surface of the
B200 attention callables the blocks use (attn.JointAttention,
blocks.SingleAttention) and compute the same thing with torch autograd on
any device, in the reference's dtypes: per-stream q/k RMSNorm (statistics in
fp32, cast, times the weight; crates/foundry-spike/src/lib.rs:45-58), axial
RoPE with fp32 arithmetic and tables rounded to the compute dtype
(lib.rs:77-129), the joint text-then-image sequence, and attention with fp32
scores and softmax, probabilities cast to the compute dtype before PV
(lib.rs:133-149). With them the block code runs on CPU and is compared with
the reference's recorded block pair (tests/golden/block_fixture.npz).

`FixtureRun` replays that block pair: double block, joint [txt, img]
sequence, single block, MSE loss, backward to the LoRA factors and the
inputs, AdamW on the LoRA factors (the generator's pipeline,
tools/fixtures/gen_block.py:297-411 in the reference).
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Dict

import numpy as np
import torch

from foundry_trainer_b200 import blocks

GOLDEN = Path(__file__).resolve().parent / "golden"
THETA = 10000.0


def rope_tables(pos: torch.Tensor, dtype) -> tuple:
    """(S, 128) cos/sin for 4 axes of 32 dims: frequency j of an axis is
    theta^(-2j/32) on both halves; fp32, then rounded to `dtype`."""
    cs, sn = [], []
    j = torch.arange(16, dtype=torch.float32)
    inv = THETA ** (-2.0 * j / 32.0)
    for a in range(4):
        f = pos[:, a:a + 1].float() * inv
        f = torch.cat([f, f], dim=-1)
        cs.append(torch.cos(f))
        sn.append(torch.sin(f))
    return torch.cat(cs, -1).to(dtype), torch.cat(sn, -1).to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    parts = []
    for a in range(4):
        seg = x[..., 32 * a:32 * (a + 1)]
        parts += [-seg[..., 16:], seg[..., :16]]
    return torch.cat(parts, -1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    c = cos.float()[None, :, None, :]
    s = sin.float()[None, :, None, :]
    return (xf * c + rotate_half(xf) * s).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = blocks.NORM_EPS) -> torch.Tensor:
    xf = x.float()
    return (xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def attention(q, k, v):
    scale = 1.0 / math.sqrt(q.shape[-1])
    qh, kh, vh = (t.transpose(1, 2) for t in (q, k, v))  # (B, H, S, D)
    p = torch.softmax((qh.float() @ kh.float().transpose(-1, -2)) * scale, dim=-1).to(q.dtype)
    return (p @ vh).transpose(1, 2)


class TorchJointAttention:
    def __init__(self, positions: torch.Tensor, dtype):
        self.cos, self.sin = rope_tables(positions, dtype)

    def __call__(self, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i):
        T = q_t.shape[1]
        q = torch.cat([rms_norm(q_t, wq_t), rms_norm(q_i, wq_i)], dim=1)
        k = torch.cat([rms_norm(k_t, wk_t), rms_norm(k_i, wk_i)], dim=1)
        v = torch.cat([v_t, v_i], dim=1)
        cos, sin = self.cos.to(q.device), self.sin.to(q.device)
        o = attention(apply_rope(q, cos, sin), apply_rope(k, cos, sin), v)
        return o[:, :T], o[:, T:]


class TorchSingleAttention:
    def __init__(self, positions: torch.Tensor, dtype):
        self.cos, self.sin = rope_tables(positions, dtype)

    def __call__(self, q, k, v, wq, wk):
        cos, sin = self.cos.to(q.device), self.sin.to(q.device)
        return attention(apply_rope(rms_norm(q, wq), cos, sin),
                         apply_rope(rms_norm(k, wk), cos, sin), v)


class Fixture:
    """tests/golden/block_fixture.npz (keys with ':' for '/')."""

    def __init__(self):
        self.z = np.load(GOLDEN / "block_fixture.npz")
        dim, heads, head_dim, rank = (int(x) for x in self.z["config"])
        self.shape = blocks.BlockShape(dim=dim, heads=heads, head_dim=head_dim)
        self.lora_scale = float(self.z["lora_scale"])
        lr, b1, b2, eps = (float(x) for x in self.z["adamw"])
        self.adamw = blocks.AdamW(lr=lr, beta1=b1, beta2=b2, eps=eps)
        self.pos_img = torch.from_numpy(self.z["pos_img"])
        self.pos_txt = torch.from_numpy(self.z["pos_txt"])

    def get(self, key: str) -> torch.Tensor:
        return torch.from_numpy(self.z[key.replace("/", ":")])

    def weights(self, dtype, device) -> Dict[str, torch.Tensor]:
        return {k.replace(":", "/"): torch.from_numpy(self.z[k]).to(device=device, dtype=dtype)
                for k in self.z.files if k.startswith("weights:")}

    def recorded(self, tag: str, key: str) -> torch.Tensor:
        return self.get(f"{tag}:{key}")


class FixtureRun:
    """The recorded pipeline on `device` in `dtype` with the given attention
    factories (positions -> callable)."""

    def __init__(self, fx: Fixture, dtype, device, joint_factory, single_factory):
        self.fx, self.dtype, self.device = fx, dtype, device
        self.w = fx.weights(dtype, device)
        self.lora = blocks.lora_keys(self.w)
        # the double block's joint sequence is [txt, img] with each stream's
        # own positions; the single block's positions are image-then-text over
        # the [txt, img] sequence, as recorded (gen_block.py:316-326)
        self.joint = joint_factory(torch.cat([fx.pos_txt, fx.pos_img], 0))
        self.single = single_factory(torch.cat([fx.pos_img, fx.pos_txt], 0))
        inp = lambda n: fx.get(f"inputs/{n}").to(device=device, dtype=dtype)
        self.img, self.txt, self.temb = inp("img")[None], inp("txt")[None], inp("temb")
        self.target_img, self.target_txt = inp("target_img")[None], inp("target_txt")[None]
        self.T = self.txt.shape[1]

    def forward(self, img, txt, acts=None):
        fx = self.fx
        img2, txt2 = blocks.double_block(self.w, img, txt, self.temb, self.joint, fx.shape,
                                         lora_scale=fx.lora_scale, acts=acts)
        joint = torch.cat([txt2, img2], dim=1)
        out = blocks.single_block(self.w, joint, self.temb, self.single, fx.shape,
                                  lora_scale=fx.lora_scale, acts=acts)
        final_txt, final_img = out[:, :self.T], out[:, self.T:]
        if acts is not None:
            acts["output/img"], acts["output/txt"] = final_img, final_txt
        loss = blocks.mse(final_img, self.target_img) + blocks.mse(final_txt, self.target_txt)
        if acts is not None:
            acts["loss"] = loss
        return loss

    def grads(self):
        """Activations, loss, d loss / d (LoRA factors, img, txt)."""
        params = [self.w[k] for k in self.lora]
        for p in params:
            p.requires_grad_(True)
        img = self.img.clone().requires_grad_(True)
        txt = self.txt.clone().requires_grad_(True)
        acts: Dict[str, torch.Tensor] = {}
        loss = self.forward(img, txt, acts)
        g = torch.autograd.grad(loss, params + [img, txt])
        out = {"grad/" + k[len("weights/"):]: v for k, v in zip(self.lora, g[:len(params)])}
        out["grad/inputs/img"], out["grad/inputs/txt"] = g[-2][0], g[-1][0]
        return acts, out

    def train(self, steps: int):
        """AdamW on the LoRA factors; returns the factors after each step."""
        params = [self.w[k] for k in self.lora]
        for p in params:
            p.requires_grad_(True)
        opt = self.fx.adamw
        state = opt.init(params)
        hist = []
        for t in range(1, steps + 1):
            loss = self.forward(self.img, self.txt)
            g = torch.autograd.grad(loss, params)
            opt.step(params, g, state, t)
            hist.append({k: p.detach().clone() for k, p in zip(self.lora, params)})
        return hist


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().flatten(), b.detach().double().flatten()
    return float((a - b).norm() / (b.norm() + 1e-12))


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().flatten(), b.detach().double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


def dp_gloo_rank(rank, world, port, steps, results):
    """One data-parallel replica of the LoRA block step on a gloo group (CPU,
    torch stand-in attention): its own seeded batch, gradients averaged by
    blocks.allreduce_mean; reports the first step's averaged gradients and
    the LoRA factors after `steps` steps."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        tr, batches = dp_problem(world)
        seen = []

        def hook(grads):
            avg = blocks.allreduce_mean(grads)
            seen.append([g.clone() for g in avg])
            return avg

        tr.grad_hook = hook
        for _ in range(steps):
            tr.step(*batches[rank])
        # numpy by value: tensors would be shared by file descriptor, which
        # dies with this process
        results.put((rank, [g.numpy() for g in seen[0]],
                     {k: p.detach().numpy().copy() for k, p in zip(tr.keys, tr.params)}))
    finally:
        dist.destroy_process_group()


def dp_problem(world):
    """A small FLUX-style block (dim 256, 2 heads) with the stand-in attention
    and one seeded batch per replica."""
    w = blocks.make_c3_weights(dim=256, heads=2, rank=4, seed=3, dtype=torch.float32)
    g = torch.Generator().manual_seed(11)
    for k in w:
        if k.endswith(".lora_b"):  # non-zero B so every factor moves from step 1
            w[k] = torch.randn(w[k].shape, generator=g) * 0.01
    pos = blocks.joint_positions(8, 4)
    tr = blocks.LoraTrainer(w, blocks.BlockShape(256, 2), pos,
                            attention=TorchJointAttention(pos, torch.float32))
    batches = []
    for r in range(world):
        gr = torch.Generator().manual_seed(100 + r)
        batches.append((torch.randn(1, 16, 256, generator=gr), torch.randn(1, 8, 256, generator=gr),
                        torch.randn(256, generator=gr), torch.randn(1, 16, 256, generator=gr),
                        torch.randn(1, 8, 256, generator=gr)))
    return tr, batches
