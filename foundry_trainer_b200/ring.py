"""Sequence-parallel (ring) attention over torch.distributed.

The reference runs the joint attention op on one GPU
(crates/foundry-spike/src/lib.rs:363-368 calls `AttnBwd` on the whole
`cat([txt, img])` sequence). At 512 + 128x128 tokens one sequence is 16896
rows; this module shards it along the sequence over the ranks of a process
group and computes the same result with one exchange pattern, a ring:

  forward   each rank keeps its query rows Q_r and passes the K/V shards
            round the ring (rank r sends to r+1, receives from r-1). At step
            t it attends its rows to shard (r - t) mod W with `fa_fwd_fold`,
            whose epilogue folds the block into fp32 (O, LSE) accumulators
            (and on the last step writes the final bf16 O and LSE); the next
            shard's transfer runs on NCCL's stream while the block computes.
  backward  K/V shards travel the same way; each shard's fp32 dK/dV
            accumulator travels one step behind it. At step t a rank writes
            the block's dK/dV to a local buffer (`fa_bwd_partial`, store
            mode) while the accumulator for that shard arrives, then adds
            the block into it (`fa_add_f32`) and passes it on; dQ stays local
            (TMA reduce-adds into a (B, H, S_pad, D) fp32 buffer). After W
            steps every accumulator has reached its owner.

Each rank holds an equal shard of S_loc = S / W rows with its own axial
positions; RoPE is applied to the local q/k before the ring starts (the K
shards travel rotated) and the gradients are un-rotated with the local
positions at the end. W = 1 runs the same code with no exchange.

The per-block arithmetic is the C ABI's (`RingKernels`); `RingComm` is the
exchange. Both are separate objects so the schedule can be checked on CPU
ranks (gloo) with a test stand-in for the kernels.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib, ops
from ._lib import check


class RingComm:
    """Neighbour exchange on a ring of the ranks of `group`."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 1:
            to_global = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
            self.next = to_global((self.rank + 1) % self.world)
            self.prev = to_global((self.rank - 1) % self.world)

    def exchange(self, send: Sequence[torch.Tensor], recv: Sequence[torch.Tensor]):
        """Start sending `send` to the next rank and receiving `recv` from the
        previous one; returns the list of works to wait on."""
        if self.world == 1:
            return []
        ops_ = [dist.P2POp(dist.isend, t, self.next, self.group) for t in send]
        ops_ += [dist.P2POp(dist.irecv, t, self.prev, self.group) for t in recv]
        return dist.batch_isend_irecv(ops_)

    @staticmethod
    def wait(works) -> None:
        for w in works:
            w.wait()


class RingKernels:
    """The per-block device calls of the ring, over the C ABI (bf16)."""

    def rope(self, x: torch.Tensor, pos: torch.Tensor, *, inverse: bool = False,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ops.rope_apply(x, ops.Rope(pos), inverse=inverse, out=out)

    def fwd_partial(self, q, k, v, scale, o_blk, lse_blk) -> None:
        B, S, H, D = q.shape
        kv_len = k.shape[1]
        dq_, dk_, dv_, do_ = ops.desc(q), ops.desc(k), ops.desc(v), ops.desc(o_blk)
        check(_lib.load().fa_fwd_partial(ops._dtype_code(q), B, S, kv_len, H, D, C.byref(dq_),
                                         C.byref(dk_), C.byref(dv_), C.byref(do_),
                                         lse_blk.data_ptr(), scale, ops._stream_ptr(None)),
              "fa_fwd_partial")

    def fwd_fold(self, q, k, v, scale, o_acc, lse_acc, step: int, last: bool, o, lse) -> None:
        B, S, H, D = q.shape
        kv_len = k.shape[1]
        dq_, dk_, dv_, do_ = ops.desc(q), ops.desc(k), ops.desc(v), ops.desc(o)
        check(_lib.load().fa_fwd_fold(ops._dtype_code(q), B, S, kv_len, H, D, C.byref(dq_),
                                      C.byref(dk_), C.byref(dv_), o_acc.data_ptr(),
                                      lse_acc.data_ptr(), step, int(last), C.byref(do_),
                                      lse.data_ptr(), scale, ops._stream_ptr(None)),
              "fa_fwd_fold")

    def lse_merge(self, o_acc, lse_acc, o_blk, lse_blk, first: bool) -> None:
        B, S, H, D = o_blk.shape
        d = ops.desc(o_blk)
        check(_lib.load().fa_lse_merge(ops._dtype_code(o_blk), B, S, H, D, o_acc.data_ptr(),
                                       lse_acc.data_ptr(), C.byref(d), lse_blk.data_ptr(),
                                       int(first), ops._stream_ptr(None)), "fa_lse_merge")

    def bwd_prepare(self, o, d_o, lse, lse2_pad, delta_pad) -> None:
        B, S, H, D = o.shape
        do_, dd_ = ops.desc(o), ops.desc(d_o)
        check(_lib.load().fa_bwd_prepare(ops._dtype_code(o), B, S, H, D, C.byref(do_),
                                         C.byref(dd_), lse.data_ptr(), lse2_pad.data_ptr(),
                                         delta_pad.data_ptr(), ops._stream_ptr(None)),
              "fa_bwd_prepare")

    def bwd_partial(self, q, k, v, d_o, lse2_pad, delta_pad, dq_acc, dk_out, dv_out, scale,
                    accumulate: bool) -> None:
        B, S, H, D = q.shape
        kv_len = k.shape[1]
        ds = [ops.desc(x) for x in (q, k, v, d_o)]
        check(_lib.load().fa_bwd_partial(ops._dtype_code(q), B, S, kv_len, H, D,
                                         *[C.byref(x) for x in ds], lse2_pad.data_ptr(),
                                         delta_pad.data_ptr(), dq_acc.data_ptr(),
                                         dk_out.data_ptr(), dv_out.data_ptr(), int(accumulate),
                                         scale, ops._stream_ptr(None)), "fa_bwd_partial")

    def add(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        check(_lib.load().fa_add_f32(dst.numel(), dst.data_ptr(), src.data_ptr(),
                                     ops._stream_ptr(None)), "fa_add_f32")

    def cast(self, x: torch.Tensor, layout: int, alpha: float, pos: Optional[torch.Tensor],
             out: torch.Tensor) -> torch.Tensor:
        B, S, H, D = out.shape
        d = ops.desc(out)
        r = ops.Rope(pos).c_struct() if pos is not None else None
        check(_lib.load().fa_cast_f32(ops._dtype_code(out), B, S, H, D, x.data_ptr(), layout,
                                      C.byref(d), alpha, C.byref(r) if r is not None else None,
                                      ops._stream_ptr(None)), "fa_cast_f32")
        return out


def _s_pad(S: int) -> int:
    return (S + 127) // 128 * 128


def ring_fwd(q, k, v, pos, scale, comm: RingComm, kern):
    """Local (O, LSE, q_rot, k_rot) of ring attention; q/k/v (B, S_loc, H, D)."""
    B, S, H, D = q.shape
    dev = q.device
    if pos is not None:
        q_r = kern.rope(q, pos)
        k_r = kern.rope(k, pos)
    else:
        q_r, k_r = q, k.contiguous()
    v_c = v.contiguous()
    o_acc = torch.empty((B, S, H, D), device=dev, dtype=torch.float32)
    lse_acc = torch.empty((B, H, S), device=dev, dtype=torch.float32)
    o = torch.empty((B, S, H, D), device=dev, dtype=q.dtype)
    lse = torch.empty((B, H, S), device=dev, dtype=torch.float32)
    bufs = [[torch.empty_like(k_r), torch.empty_like(v_c)] for _ in range(2)] if comm.world > 1 else []
    cur = [k_r, v_c]
    for t in range(comm.world):
        works = []
        if t < comm.world - 1:
            nxt = bufs[t % 2]
            works = comm.exchange(cur, nxt)
        # the block folds into (o_acc, lse_acc) inside the kernel; the last
        # block writes the final o and lse
        kern.fwd_fold(q_r, cur[0], cur[1], scale, o_acc, lse_acc, t, t == comm.world - 1, o, lse)
        if t < comm.world - 1:
            comm.wait(works)
            cur = nxt
    return o, lse, q_r, k_r


def ring_bwd(q_r, k_r, v, o, d_o, lse, pos, scale, comm: RingComm, kern):
    """Local (dq, dk, dv) of ring attention w.r.t. the pre-rotation q/k."""
    B, S, H, D = q_r.shape
    dev = q_r.device
    sp = _s_pad(S)
    lse2_pad = torch.empty((B, H, sp), device=dev, dtype=torch.float32)
    delta_pad = torch.empty((B, H, sp), device=dev, dtype=torch.float32)
    kern.bwd_prepare(o, d_o, lse, lse2_pad, delta_pad)
    dq_acc = torch.zeros((B, H, sp, D), device=dev, dtype=torch.float32)
    v_c = v.contiguous()
    W = comm.world
    # accumulators: [dK | dV] fp32, one travelling buffer pair plus a block buffer
    acc = [torch.empty((2, B, S, H, D), device=dev, dtype=torch.float32) for _ in range(2 if W > 1 else 1)]
    part = torch.empty((2, B, S, H, D), device=dev, dtype=torch.float32) if W > 1 else None
    kv_bufs = [[torch.empty_like(k_r), torch.empty_like(v_c)] for _ in range(2)] if W > 1 else []
    cur_kv = [k_r, v_c]
    a_cur = 0
    acc_works: List = []
    for t in range(W):
        kv_works = []
        if t < W - 1:
            nxt_kv = kv_bufs[t % 2]
            kv_works = comm.exchange(cur_kv, nxt_kv)
        if t == 0:
            kern.bwd_partial(q_r, cur_kv[0], cur_kv[1], d_o, lse2_pad, delta_pad, dq_acc,
                             acc[a_cur][0], acc[a_cur][1], scale, False)
        else:
            kern.bwd_partial(q_r, cur_kv[0], cur_kv[1], d_o, lse2_pad, delta_pad, dq_acc,
                             part[0], part[1], scale, False)
            comm.wait(acc_works)
            kern.add(acc[a_cur], part)
        if W > 1:
            # pass the shard's accumulator on; after the last step it reaches its owner
            acc_works = comm.exchange([acc[a_cur]], [acc[1 - a_cur]])
            a_cur = 1 - a_cur
        if t < W - 1:
            comm.wait(kv_works)
            cur_kv = nxt_kv
    comm.wait(acc_works)
    final = acc[a_cur]
    dq = kern.cast(dq_acc, 1, scale, pos, torch.empty((B, S, H, D), device=dev, dtype=q_r.dtype))
    dk = kern.cast(final[0], 0, 1.0, pos, torch.empty((B, S, H, D), device=dev, dtype=q_r.dtype))
    dv = kern.cast(final[1], 0, 1.0, None, torch.empty((B, S, H, D), device=dev, dtype=q_r.dtype))
    return dq, dk, dv


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, pos, scale, comm, kern):
        o, lse, q_r, k_r = ring_fwd(q, k, v, pos, scale, comm, kern)
        ctx.save_for_backward(q_r, k_r, v, o, lse)
        ctx.pos, ctx.scale, ctx.comm, ctx.kern = pos, scale, comm, kern
        return o

    @staticmethod
    def backward(ctx, grad_o):
        q_r, k_r, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ring_bwd(q_r, k_r, v, o, grad_o.contiguous(), lse, ctx.pos, ctx.scale,
                              ctx.comm, ctx.kern)
        return dq, dk, dv, None, None, None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                   pos: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                   group=None, comm: Optional[RingComm] = None, kernels=None) -> torch.Tensor:
    """Attention of this rank's rows (B, S_loc, H, D) against the whole
    sequence held across the ring; differentiable. `pos` are this shard's
    (S_loc, 4) axial positions (RoPE applied inside), or None for no RoPE.
    Every rank of the group must call it with the same S_loc."""
    q4, k4, v4 = ops.as_bshd(q), ops.as_bshd(k), ops.as_bshd(v)
    if k4.shape != q4.shape or v4.shape != q4.shape:
        raise ValueError("q, k, v shards must share one shape")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share one dtype")
    comm = comm if comm is not None else RingComm(group)
    kern = kernels if kernels is not None else RingKernels()
    scale = ops.default_scale(q4.shape[-1]) if scale is None else float(scale)
    o = _RingAttention.apply(q4, k4, v4, pos, scale, comm, kern)
    return o if q.dim() == 4 else o.squeeze(0)
