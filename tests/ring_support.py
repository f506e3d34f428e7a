"""Test support for ring attention: CPU stand-in kernels, a threaded one-GPU
ring, and the rank workers the multi-process tests spawn.

TEST INFRASTRUCTURE ONLY. `FakeRingKernels` has the method surface of
`foundry_trainer_b200.ring.RingKernels` and computes each block with float64
torch arithmetic on CPU tensors, in the conventions of the C ABI calls it
stands in for (fa_fwd_partial, fa_lse_merge, fa_bwd_prepare, fa_bwd_partial,
fa_add_f32, fa_cast_f32): dq_acc holds the unscaled dS K in (B, H, S_pad, D),
dK is scaled in the block, lse2 = LSE * log2(e) padded with +inf. With it the
ring schedule (which shard is where at each step, the merge, the travelling
dK/dV accumulators) runs on gloo ranks without a GPU and is compared with the
single-sequence oracle.
"""
from __future__ import annotations

import math
import os
import threading
from datetime import timedelta

import numpy as np
import torch

from oracle import attn_oracle as orc

LOG2E = 1.0 / math.log(2.0)


def _rope_np(x: torch.Tensor, pos: torch.Tensor, inverse: bool) -> torch.Tensor:
    cos, sin = orc.rope_tables(pos.numpy(), "f32")
    f = orc.apply_rope_grad if inverse else orc.apply_rope
    return torch.from_numpy(np.stack([f(xb, cos, sin, "f32") for xb in x.float().numpy()]))


class FakeRingKernels:
    def __init__(self):
        self.calls = []

    def rope(self, x, pos, *, inverse=False, out=None):
        self.calls.append("rope")
        y = _rope_np(x, pos, inverse).to(x.dtype)
        if out is None:
            return y
        out.copy_(y)
        return out

    def fwd_partial(self, q, k, v, scale, o_blk, lse_blk):
        self.calls.append("fwd_partial")
        qd, kd, vd = (t.double().permute(0, 2, 1, 3) for t in (q, k, v))  # (B,H,S,D)
        s = qd @ kd.transpose(-1, -2) * scale
        lse = torch.logsumexp(s, dim=-1)
        p = torch.exp(s - lse[..., None])
        o_blk.copy_((p @ vd).permute(0, 2, 1, 3))
        lse_blk.copy_(lse)

    def fwd_fold(self, q, k, v, scale, o_acc, lse_acc, step, last, o, lse):
        """fa_fwd_fold: a block folded into (o_acc, lse_acc); the last writes o, lse."""
        B, S, H, D = q.shape
        o_blk = torch.empty((B, S, H, D), dtype=torch.float64)
        lse_blk = torch.empty((B, H, S), dtype=torch.float64)
        self.fwd_partial(q, k, v, scale, o_blk, lse_blk)
        if step == 0 and last:
            o.copy_(o_blk)
            lse.copy_(lse_blk)
            return
        if step == 0:
            o_acc.copy_(o_blk)
            lse_acc.copy_(lse_blk)
            return
        self.lse_merge(o_acc, lse_acc, o_blk, lse_blk, False)
        if last:
            o.copy_(o_acc)
            lse.copy_(lse_acc)

    def lse_merge(self, o_acc, lse_acc, o_blk, lse_blk, first):
        self.calls.append("lse_merge")
        if first:
            o_acc.copy_(o_blk)
            lse_acc.copy_(lse_blk)
            return
        la, lb = lse_acc.double(), lse_blk.double()
        m = torch.maximum(la, lb)
        wa, wb = torch.exp(la - m), torch.exp(lb - m)
        tr = lambda w: w.permute(0, 2, 1)[..., None]  # (B,H,S) -> (B,S,H,1)
        o_acc.copy_((o_acc.double() * tr(wa) + o_blk.double() * tr(wb)) / tr(wa + wb))
        lse_acc.copy_(m + torch.log(wa + wb))

    def bwd_prepare(self, o, d_o, lse, lse2_pad, delta_pad):
        self.calls.append("bwd_prepare")
        S = o.shape[1]
        lse2_pad.fill_(float("inf"))
        delta_pad.zero_()
        lse2_pad[:, :, :S] = lse * LOG2E
        delta_pad[:, :, :S] = (o.double() * d_o.double()).sum(-1).permute(0, 2, 1)

    def bwd_partial(self, q, k, v, d_o, lse2_pad, delta_pad, dq_acc, dk_out, dv_out, scale,
                    accumulate):
        self.calls.append("bwd_partial")
        S = q.shape[1]
        qd, kd, vd, dod = (t.double().permute(0, 2, 1, 3) for t in (q, k, v, d_o))
        s2 = qd @ kd.transpose(-1, -2) * (scale * LOG2E)
        p = torch.exp2(s2 - lse2_pad[:, :, :S, None].double())
        dp = dod @ vd.transpose(-1, -2)
        ds = p * (dp - delta_pad[:, :, :S, None].double())
        dq_acc[:, :, :S] += (ds @ kd).float()
        dk = (scale * ds.transpose(-1, -2) @ qd).permute(0, 2, 1, 3)
        dv = (p.transpose(-1, -2) @ dod).permute(0, 2, 1, 3)
        if accumulate:
            dk_out += dk.float()
            dv_out += dv.float()
        else:
            dk_out.copy_(dk)
            dv_out.copy_(dv)

    def add(self, dst, src):
        self.calls.append("add")
        dst += src

    def cast(self, x, layout, alpha, pos, out):
        self.calls.append("cast")
        S = out.shape[1]
        y = x[:, :, :S].permute(0, 2, 1, 3) if layout == 1 else x
        y = y.double() * alpha
        if pos is not None:
            y = _rope_np(y.float(), pos, inverse=True).double()
        out.copy_(y)
        return out


def full_problem(B, S, H, D, seed):
    """Seeded f32 (q, k, v, d_o) of the whole sequence and its axial positions."""
    g = torch.Generator().manual_seed(seed)
    q, k, v, d_o = (torch.randn((B, S, H, D), generator=g) * 0.5 for _ in range(4))
    grid = int(math.isqrt(S))
    txt = S - grid * grid
    pos = torch.zeros((S, 4))
    i = torch.arange(grid * grid)
    pos[txt:, 1] = (i // grid).float()
    pos[txt:, 2] = (i % grid).float()
    return q, k, v, d_o, pos


def gloo_rank(rank, world, port, shape, seed, results):
    """One gloo rank: ring attention of its shard with the CPU stand-in."""
    import torch.distributed as dist

    from foundry_trainer_b200 import ring

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, S, H, D = shape
        q, k, v, d_o, pos = full_problem(B, S, H, D, seed)
        n = S // world
        sl = slice(rank * n, (rank + 1) * n)
        qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        kern = FakeRingKernels()
        o = ring.ring_attention(qs, ks, vs, pos=pos[sl].contiguous(), kernels=kern)
        o.backward(d_o[:, sl])
        results.put((rank, o.detach().numpy(), qs.grad.numpy(), ks.grad.numpy(),
                     vs.grad.numpy(), kern.calls))
    finally:
        dist.destroy_process_group()


class ThreadRing:
    """W ranks of a ring as W threads of one process on one GPU.

    `comm(rank)` returns an object with RingComm's surface whose exchange
    copies, between two barriers, what the previous rank offered into the
    receive buffers. All threads enqueue on the one default stream, so the
    copies run after the kernels that produced their sources.
    """

    def __init__(self, world: int):
        self.world = world
        self.slots = [None] * world
        self.barrier = threading.Barrier(world, timeout=120)

    def comm(self, rank: int):
        ring = self

        class _Comm:
            world = ring.world

            def exchange(self, send, recv):
                ring.slots[rank] = list(send)
                ring.barrier.wait()
                for dst, src in zip(recv, ring.slots[(rank - 1) % ring.world]):
                    dst.copy_(src)
                ring.barrier.wait()
                return []

            @staticmethod
            def wait(works):
                pass

        return _Comm()


def nccl_rank(rank, world, port, arrays, results):
    """One NCCL rank on cuda:rank: bf16 ring attention of its shard."""
    import torch.distributed as dist

    from foundry_trainer_b200 import ops, ring

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        q, k, v, d_o, pos = (torch.from_numpy(a) for a in arrays)
        n = q.shape[1] // world
        sl = slice(rank * n, (rank + 1) * n)
        to = lambda t: t[:, sl].to(torch.bfloat16).cuda().requires_grad_(True)
        qs, ks, vs = to(q), to(k), to(v)
        o = ring.ring_attention(qs, ks, vs, pos=pos[sl].contiguous().cuda())
        o.backward(d_o[:, sl].to(torch.bfloat16).cuda())
        torch.cuda.synchronize()
        status = ops.device_status()
        f = lambda t: t.detach().float().cpu().numpy()
        results.put((rank, f(o), f(qs.grad), f(ks.grad), f(vs.grad), status))
    finally:
        dist.destroy_process_group()
