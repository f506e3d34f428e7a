"""Test infrastructure for the head-parallel schedule (foundry_trainer_b200/heads.py).

`FakeHeadKernels` stands in for the C ABI on CPU ranks: the forward and
backward of one head group over the whole sequence from the fp32 oracle
(RoPE at the given positions), so a gloo run checks the exchange layout and
the schedule, not the kernels. `gloo_rank` is one rank of such a run;
`nccl_rank` one rank of the real path on its own GPU.
"""
import os

import numpy as np
import torch

from oracle import attn_oracle as orc
from tests.ring_support import full_problem


class FakeHeadKernels:
    """HeadKernels' surface computed by the oracle (fp32 numpy)."""

    def __init__(self):
        self.calls = []

    def fwd(self, q, k, v, pos, scale):
        self.calls.append(("fwd", tuple(q.shape)))
        z = np.zeros(q.shape, np.float32)
        o, lse, _, _, _ = orc.attn_fwd_bwd_bshd(q.numpy(), k.numpy(), v.numpy(), z, "f32",
                                                rope_pos=pos.numpy() if pos is not None else None)
        return torch.from_numpy(np.ascontiguousarray(o)), torch.from_numpy(lse), pos

    def bwd(self, q, k, v, o, d_o, lse, scale, ctx):
        self.calls.append(("bwd", tuple(q.shape)))
        pos = ctx
        _, _, dq, dk, dv = orc.attn_fwd_bwd_bshd(q.numpy(), k.numpy(), v.numpy(), d_o.numpy(),
                                                 "f32",
                                                 rope_pos=pos.numpy() if pos is not None else None)
        return tuple(torch.from_numpy(np.ascontiguousarray(x)) for x in (dq, dk, dv))


def gloo_rank(rank, world, port, shape, seed, results):
    """One gloo rank: the head-parallel op on its sequence shard, under autograd."""
    import torch.distributed as dist

    from foundry_trainer_b200 import heads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, S, H, D = shape
        q, k, v, d_o, pos = full_problem(B, S, H, D, seed)
        n = S // world
        sl = slice(rank * n, (rank + 1) * n)
        qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        kern = FakeHeadKernels()
        o = heads.head_parallel_attention(qs, ks, vs, pos=pos, kern=kern)
        o.backward(d_o[:, sl])
        results.put((rank, o.detach().numpy(), qs.grad.numpy(), ks.grad.numpy(),
                     vs.grad.numpy(), kern.calls))
    finally:
        dist.destroy_process_group()


def nccl_rank(rank, world, port, arrays, results, steps):
    """One rank on GPU `rank`: the head-parallel schedule with the real
    kernels and NCCL all-to-alls, `steps` times; returns the last step's
    shards of O, dQ, dK, dV and the device status word."""
    import torch.distributed as dist

    from foundry_trainer_b200 import heads, ops

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        q, k, v, d_o, pos = (torch.from_numpy(a) for a in arrays)
        n = q.shape[1] // world
        sl = slice(rank * n, (rank + 1) * n)
        dev = torch.device("cuda", rank)
        qs, ks, vs, dos = (t[:, sl].to(torch.bfloat16).contiguous().to(dev)
                           for t in (q, k, v, d_o))
        pos_d = pos.contiguous().to(dev)
        ex, kern = heads.HeadExchange(), heads.HeadKernels()
        scale = ops.default_scale(q.shape[-1])
        for _ in range(steps):
            o, state = heads.head_fwd(qs, ks, vs, pos_d, scale, ex, kern)
            dq, dk, dv = heads.head_bwd(dos, state, scale, ex, kern)
        torch.cuda.synchronize()
        f = lambda t: t.float().cpu().numpy()
        results.put((rank, f(o), f(dq), f(dk), f(dv), ops.device_status()))
    finally:
        dist.destroy_process_group()
