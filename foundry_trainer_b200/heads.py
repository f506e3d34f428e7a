"""Head-parallel sequence sharding of the joint attention (all-to-all).

The reference runs the op on one GPU over the whole `cat([txt, img])`
sequence (crates/foundry-spike/src/lib.rs:363-368 calls `AttnBwd`). Here
the sequence arrives sharded: rank r holds rows [r*S_loc, (r+1)*S_loc) of
q, k, v (and later dO) for all H heads. Attention mixes every row with
every row but never one head with another, so one all-to-all turns the
sequence shards into head groups — rank r then holds the whole sequence of
heads [r*H/W, (r+1)*H/W) — and each rank runs the single-GPU op on its
heads: the forward with the axial RoPE inside its tile loads over the full
sequence (`ops.attn_fwd`, `fa_fwd`) and the backward reusing its rotated
q, k (`ops.attn_bwd(saved=...)`, `fa_bwd_saved`). A second all-to-all
returns O (and in the backward dQ, dK, dV) to the sequence layout. The
results are those of the single-GPU op on the same heads: no partial
softmax merges, no cross-rank accumulation.

Per rank and step the exchange moves (W-1)/W of its q, k, v, O, dO, dQ,
dK, dV shards (bf16) — at C5 over 8 GPUs ~90 MB each way — while the
sequence-parallel peer path moves every K/V shard to every rank and every
fp32 dK/dV contribution to its owner. The head count must divide by the
rank count (C5: 24 heads over 2, 4 or 8 ranks).

The exchange is `HeadExchange` (torch.distributed all_to_all_single on a
process group: NCCL on GPUs, gloo in the CPU tests); the per-head-group
arithmetic is `HeadKernels` (the C ABI through `ops`). Both are separate
objects so the schedule can be checked on CPU ranks with a stand-in for
the kernels.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import ops


class HeadExchange:
    """all-to-all over the ranks of `group` (sequence shards <-> head groups)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_to_all(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        """recv[i] <- rank i's send[self.rank] (equal splits of dim 0; both
        contiguous)."""
        if self.world == 1:
            recv.copy_(send)
        else:
            dist.all_to_all_single(recv, send, group=self.group)


def seq_to_heads(xs: Sequence[torch.Tensor], ex: HeadExchange) -> List[torch.Tensor]:
    """(B, S_loc, H, D) sequence shards -> (B, W*S_loc, H/W, D): this rank's
    head group over the whole sequence. One exchange per tensor: the send
    side regroups the shard by destination (one copy); with B = 1 the
    received blocks already are the head group's rows in order, so they land
    in the result without a second copy."""
    W = ex.world
    outs = []
    for x in xs:
        B, S_loc, H, D = x.shape
        if H % W:
            raise ValueError(f"{H} heads do not split over {W} ranks")
        hw = H // W
        send = x.reshape(B, S_loc, W, hw, D).permute(2, 0, 1, 3, 4).contiguous()
        y = torch.empty((B, W * S_loc, hw, D), device=x.device, dtype=x.dtype)
        if B == 1:
            ex.all_to_all(y.view(W, B, S_loc, hw, D), send)
        else:
            recv = torch.empty_like(send)
            ex.all_to_all(recv, send)
            y.view(B, W, S_loc, hw, D).copy_(recv.permute(1, 0, 2, 3, 4))
        outs.append(y)
    return outs


def heads_to_seq(xs: Sequence[torch.Tensor], ex: HeadExchange) -> List[torch.Tensor]:
    """Inverse of seq_to_heads: (B, W*S_loc, H/W, D) head groups ->
    (B, S_loc, H, D) this rank's sequence shard of all heads (with B = 1 the
    send blocks are contiguous row ranges: one copy, on the receive side)."""
    W = ex.world
    outs = []
    for x in xs:
        B, S, hw, D = x.shape
        S_loc = S // W
        if B == 1:
            send = x.reshape(W, B, S_loc, hw, D)
        else:
            send = x.reshape(B, W, S_loc, hw, D).permute(1, 0, 2, 3, 4).contiguous()
        recv = torch.empty((W, B, S_loc, hw, D), device=x.device, dtype=x.dtype)
        ex.all_to_all(recv, send)
        y = torch.empty((B, S_loc, W * hw, D), device=x.device, dtype=x.dtype)
        y.view(B, S_loc, W, hw, D).copy_(recv.permute(1, 2, 0, 3, 4))
        outs.append(y)
    return outs


class HeadKernels:
    """The single-GPU op on one head group (the C ABI through `ops`)."""

    def fwd(self, q, k, v, pos, scale):
        """(O, LSE, ctx) with the RoPE of `pos` inside (None: no RoPE); ctx
        is what bwd needs (the forward's workspace with rotated q, k)."""
        rope = ops.Rope(pos) if pos is not None else None
        saved = {}
        o, lse = ops.attn_fwd(q, k, v, scale=scale, rope=rope, saved=saved)
        return o, lse, (rope, saved)

    def bwd(self, q, k, v, o, d_o, lse, scale, ctx):
        rope, saved = ctx
        return ops.attn_bwd(q, k, v, o, d_o, lse, scale=scale, rope=rope, saved=saved)


def head_fwd(q, k, v, pos, scale, ex: HeadExchange, kern):
    """(o, state) for this rank's sequence shard; q, k, v (B, S_loc, H, D),
    pos the (S, n_axes) positions of the WHOLE sequence (None: no RoPE).
    `state` holds what head_bwd needs."""
    qh, kh, vh = seq_to_heads([q, k, v], ex)
    oh, lse, ctx = kern.fwd(qh, kh, vh, pos, scale)
    (o,) = heads_to_seq([oh], ex)
    return o, (qh, kh, vh, oh, lse, ctx)


def head_bwd(d_o, state, scale, ex: HeadExchange, kern):
    """(dq, dk, dv) of this rank's sequence shard (w.r.t. pre-rotation q, k)."""
    qh, kh, vh, oh, lse, ctx = state
    (doh,) = seq_to_heads([d_o], ex)
    dqh, dkh, dvh = kern.bwd(qh, kh, vh, oh, doh, lse, scale, ctx)
    dq, dk, dv = heads_to_seq([dqh, dkh, dvh], ex)
    return dq, dk, dv


class _HeadAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, pos, scale, ex, kern):
        o, state = head_fwd(q, k, v, pos, scale, ex, kern)
        ctx.state, ctx.scale, ctx.ex, ctx.kern = state, scale, ex, kern
        return o

    @staticmethod
    def backward(ctx, grad_o):
        dq, dk, dv = head_bwd(grad_o.contiguous(), ctx.state, ctx.scale, ctx.ex, ctx.kern)
        ctx.state = None
        return dq, dk, dv, None, None, None, None


def head_parallel_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                            pos: Optional[torch.Tensor], scale: Optional[float] = None,
                            ex: Optional[HeadExchange] = None, kern=None) -> torch.Tensor:
    """The op over a sequence sharded along S (this rank's rows), under
    autograd. `pos`: positions of the whole sequence."""
    ex = ex if ex is not None else HeadExchange()
    kern = kern if kern is not None else HeadKernels()
    scale = ops.default_scale(q.shape[-1]) if scale is None else float(scale)
    return _HeadAttention.apply(q, k, v, pos, scale, ex, kern)
