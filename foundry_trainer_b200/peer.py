"""Sequence-parallel attention over the GPUs' peer memory (one node).

The same decomposition as `ring.py` (each rank keeps S_loc query rows and
needs every K/V shard; every rank's rows contribute to every shard's dK/dV),
with the exchange done by the hardware instead of send/recv kernels:

  forward   each rank rotates its K shard into a buffer its peers can map
            (CUDA IPC), copies V beside it, and after one barrier the copy
            engine pulls the W-1 remote shards in ring order (r-1, r-2, ...)
            into a local
            (B, W*S_loc, H, D) K/V laid out in that order. The own shard is
            folded first, then the pulled ones two slots per launch as they
            land, into two fp32 (O, LSE) accumulators on two streams (so two
            launches of S_loc/256 x H CTAs share the SMs); a final merge
            writes O and LSE. Copy engines need no SMs, so the pulls run
            under the attention kernels.
  backward  the gathered K/V are reused: one `fa_bwd_scatter` launch over all
            W*S_loc keys, whose epilogue stores each key row's fp32 dK/dV
            straight into the receive slot of the rank that owns the row (a
            peer store over NVLink); dQ stays local. After one barrier each
            owner sums its W slots, un-rotates dK and casts
            (`fa_reduce_cast_f32`).

Two barriers per forward+backward order everything (see `PeerExchange`):
the forward's (shards published) and the backward's (contributions
delivered). Buffers peers touch are double-buffered by call parity, so one
barrier per call is enough for calls that follow one another. Within one
forward+backward pair the backward's barrier already orders the next
forward's writes after every peer's reads (and the forward's barrier the
next backward's stores after the owner's sum), so a CUDA graph of one pair,
replayed with its captured parity, is also safe.

The reference runs the op on one device (crates/foundry-spike/src/lib.rs
:189-263); this path is the long-sequence configuration's multi-GPU form and
computes the same O, dQ, dK, dV.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib, ops
from ._lib import check

_ALIGN = 4096
_SM_COPY_CTAS = 148  # one small copy CTA per SM of a B200


def _align(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


def block_order(rank: int, world: int) -> List[int]:
    """Shards in the order the forward folds them: its own, then r-1, r-2, ..."""
    return [(rank - t) % world for t in range(world)]


class Layout:
    """Byte offsets of one rank's peer allocation (identical on every rank):
    [flags | pub(2 parities) | recv(2 parities)] with
      pub[par]  = K | V of this rank's shard, bf16 (B, S, H, D) each;
      recv[par] = (W, 2, B, S, H, D) fp32: slot src, 0 = dK, 1 = dV, the
                  contributions of rank src's query rows to this rank's keys.
    """

    def __init__(self, B: int, S: int, H: int, D: int, world: int, flags_bytes: int):
        self.n = B * S * H * D
        self.world = world
        self.flags = 0
        self.pub = _align(flags_bytes)
        self.pub_bytes = 2 * self.n * 2
        self.recv = _align(self.pub + 2 * self.pub_bytes)
        self.recv_bytes = world * 2 * self.n * 4
        self.total = _align(self.recv + 2 * self.recv_bytes)

    def pub_off(self, par: int, which: int) -> int:
        return self.pub + par * self.pub_bytes + which * self.n * 2

    def recv_off(self, par: int, src: int, which: int) -> int:
        return self.recv + par * self.recv_bytes + (src * 2 + which) * self.n * 4


class _DevView:
    """`__cuda_array_interface__` of a raw device range (zero-copy tensors)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "strides": None, "version": 2}


def _tensor_at(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    typestr = {torch.bfloat16: "<i2", torch.float32: "<f4"}[dtype]
    t = torch.as_tensor(_DevView(ptr, shape, typestr), device=device)
    return t.view(dtype) if dtype == torch.bfloat16 else t


class PeerExchange:
    """Peer buffers, barriers and copy streams of the ranks of `group` for
    shards of shape (B, S, H, D) bf16. All ranks must be on one node and
    construct it together (the IPC handles are exchanged over the group)."""

    def __init__(self, B: int, S: int, H: int, D: int, *, group=None, timeout_s: float = 30.0,
                 device: Optional[torch.device] = None, copy: str = "ce"):
        self.group = group
        dist_on = dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if self.world > 8:
            raise ValueError("the peer exchange spans at most 8 ranks (one node)")
        if copy not in ("ce", "sm"):
            raise ValueError("copy must be 'ce' (copy engines) or 'sm' (a copy kernel)")
        self.copy = copy
        self.shape = (B, S, H, D)
        self.device = device if device is not None else torch.device("cuda",
                                                                     torch.cuda.current_device())
        self.timeout_s = float(timeout_s)
        lib = _lib.load()
        self.lay = Layout(B, S, H, D, self.world, int(lib.fa_peer_flags_bytes()))
        ptr, handle = C.c_void_p(), _lib.fa_peer_handle_t()
        check(lib.fa_peer_alloc(self.lay.total, C.byref(ptr), C.byref(handle)), "fa_peer_alloc")
        self._own = ptr.value
        self._opened: List[int] = []
        bases = [0] * self.world
        bases[self.rank] = self._own
        if self.world > 1:
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.bytes), group=group)
            for p in range(self.world):
                if p == self.rank:
                    continue
                h = _lib.fa_peer_handle_t()
                C.memmove(h.bytes, handles[p], 64)
                q = C.c_void_p()
                check(lib.fa_peer_open(C.byref(h), C.byref(q)), "fa_peer_open")
                bases[p] = q.value
                self._opened.append(q.value)
        self.bases = bases
        self._flags = (C.c_void_p * self.world)(*[b + self.lay.flags for b in bases])
        # one copy stream: copies on several streams share one copy engine
        # and are served stream after stream, not in issue order
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.side_stream = torch.cuda.Stream(device=self.device)
        self.n_fwd = 0
        self.n_bwd = 0
        if self.world > 1:
            dist.barrier(group=group)  # every rank has mapped every other

    # -- views and addresses
    def pub(self, par: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return tuple(_tensor_at(self._own + self.lay.pub_off(par, w), self.shape, torch.bfloat16,
                                self.device) for w in (0, 1))

    def recv(self, par: int) -> torch.Tensor:
        return _tensor_at(self._own + self.lay.recv_off(par, 0, 0),
                          (self.world, 2) + self.shape, torch.float32, self.device)

    def recv_ptrs(self, par: int, which: int) -> List[int]:
        """Where this rank's contribution to each owner's keys goes."""
        return [self.bases[o] + self.lay.recv_off(par, self.rank, which)
                for o in range(self.world)]

    # -- operations (stream ordered)
    def barrier(self, channel: int, stream=None) -> None:
        check(_lib.load().fa_peer_barrier(self.rank, self.world, self._flags, channel,
                                          self.timeout_s, ops._stream_ptr(stream)),
              "fa_peer_barrier")

    def pull(self, par: int, src: int, slot: int, which: int, dst: torch.Tensor,
             stream) -> None:
        """Copies rank src's published K (which 0) or V (1) shard into rows
        [slot*S, (slot+1)*S) of dst ((B, W*S, H, D) contiguous) on `stream`."""
        B, S, H, D = self.shape
        row = S * H * D * 2
        src_ptr = self.bases[src] + self.lay.pub_off(par, which)
        lib = _lib.load()
        if self.copy == "sm":
            check(lib.fa_copy_2d_sm(dst.data_ptr() + slot * row, self.world * row, src_ptr, row,
                                    row, B, _SM_COPY_CTAS, ops._stream_ptr(stream)),
                  "fa_copy_2d_sm")
        else:
            check(lib.fa_copy_2d(dst.data_ptr() + slot * row, self.world * row, src_ptr, row,
                                 row, B, ops._stream_ptr(stream)), "fa_copy_2d")

    def check(self) -> None:
        """Raises FaError(FA_ERR_DEVICE_TIMEOUT) when a bounded device wait
        on this device expired since the last check, i.e. a peer did not
        reach a barrier in time: its shard or its dK/dV contributions are
        missing and the step's results are wrong. Synchronises the device
        (and clears the status word)."""
        check(ops.device_status(), "peer exchange (a peer missed a barrier)")

    def close(self) -> None:
        """Unmaps the peers and frees this rank's buffer (all ranks together)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        lib = _lib.load()
        for p in self._opened:
            lib.fa_peer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)  # nobody maps this buffer any more
        lib.fa_peer_free(self._own)
        self._own = None


class PeerKernels:
    """The device calls of the peer path, over the C ABI (bf16)."""

    def rope(self, x, pos, *, out=None):
        return ops.rope_apply(x, ops.Rope(pos), out=out)

    def fwd_fold(self, q, k, v, scale, o_acc, lse_acc, step, last, o, lse, stream=None):
        B, S, H, D = q.shape
        d = [ops.desc(x) for x in (q, k, v, o)]
        check(_lib.load().fa_fwd_fold(ops._dtype_code(q), B, S, k.shape[1], H, D,
                                      *[C.byref(x) for x in d[:3]], o_acc.data_ptr(),
                                      lse_acc.data_ptr(), step, int(last), C.byref(d[3]),
                                      lse.data_ptr(), scale, ops._stream_ptr(stream)),
              "fa_fwd_fold")

    def merge(self, o_a, lse_a, o_b, lse_b, o, lse, stream=None):
        B, S, H, D = o.shape
        d = ops.desc(o)
        check(_lib.load().fa_merge_f32(ops._dtype_code(o), B, S, H, D, o_a.data_ptr(),
                                       lse_a.data_ptr(), o_b.data_ptr(), lse_b.data_ptr(),
                                       C.byref(d), lse.data_ptr(), ops._stream_ptr(stream)),
              "fa_merge_f32")

    def bwd_prepare(self, o, d_o, lse, lse2_pad, delta_pad):
        B, S, H, D = o.shape
        do_, dd_ = ops.desc(o), ops.desc(d_o)
        check(_lib.load().fa_bwd_prepare(ops._dtype_code(o), B, S, H, D, C.byref(do_),
                                         C.byref(dd_), lse.data_ptr(), lse2_pad.data_ptr(),
                                         delta_pad.data_ptr(), ops._stream_ptr(None)),
              "fa_bwd_prepare")

    def bwd_scatter(self, q, k_all, v_all, d_o, lse2_pad, delta_pad, dq_acc, seg,
                    dk_ptrs, dv_ptrs, scale):
        B, S, H, D = q.shape
        d = [ops.desc(x) for x in (q, k_all, v_all, d_o)]
        n = len(dk_ptrs)
        dk_arr = (C.c_void_p * n)(*dk_ptrs)
        dv_arr = (C.c_void_p * n)(*dv_ptrs)
        check(_lib.load().fa_bwd_scatter(ops._dtype_code(q), B, S, k_all.shape[1], H, D,
                                         *[C.byref(x) for x in d], lse2_pad.data_ptr(),
                                         delta_pad.data_ptr(), dq_acc.data_ptr(), seg, n,
                                         dk_arr, dv_arr, scale, ops._stream_ptr(None)),
              "fa_bwd_scatter")

    def reduce_cast(self, recv, pos, dk, dv):
        """dk = inverse_rope(sum_p recv[p, 0]), dv = sum_p recv[p, 1]."""
        W = recv.shape[0]
        B, S, H, D = dk.shape
        r = ops.Rope(pos).c_struct() if pos is not None else None
        dk_, dv_ = ops.desc(dk), ops.desc(dv)
        check(_lib.load().fa_reduce_cast_f32(ops._dtype_code(dk), B, S, H, D, recv[0, 0].data_ptr(),
                                             recv[0, 1].data_ptr(), W, 2 * B * S * H * D,
                                             C.byref(dk_), C.byref(dv_), 1.0,
                                             C.byref(r) if r is not None else None,
                                             ops._stream_ptr(None)), "fa_reduce_cast_f32")

    def cast(self, x, layout, alpha, pos, out):
        B, S, H, D = out.shape
        d = ops.desc(out)
        r = ops.Rope(pos).c_struct() if pos is not None else None
        check(_lib.load().fa_cast_f32(ops._dtype_code(out), B, S, H, D, x.data_ptr(), layout,
                                      C.byref(d), alpha, C.byref(r) if r is not None else None,
                                      ops._stream_ptr(None)), "fa_cast_f32")
        return out


def fold_groups(world: int) -> List[List[int]]:
    """Slots of the gathered K/V folded per launch: this rank's own shard
    alone (it is ready first), then the pulled shards two at a time (two
    adjacent slots are one contiguous key range)."""
    groups = [[0]]
    t = 1
    while t < world:
        groups.append(list(range(t, min(t + 2, world))))
        t += 2
    return groups


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def _mark(trace: Optional[list], name: str, stream=None) -> None:
    """Appends (name, timing event recorded on `stream`) when tracing (inside
    a CUDA-graph capture the event becomes a record node of the graph)."""
    if trace is not None:
        e = torch.cuda.Event(enable_timing=True, external=_capturing())
        e.record(stream if stream is not None else torch.cuda.current_stream())
        trace.append((name, e))


def peer_fwd(q, k, v, pos, scale, ex: PeerExchange, kern: PeerKernels,
             trace: Optional[list] = None, check_status: bool = True):
    """(O, LSE, q_rot, k_all, v_all) of this rank's rows; q/k/v (B, S_loc, H, D)
    bf16, pos the shard's (S_loc, 4) positions (None: no RoPE). k_all / v_all
    (B, W*S_loc, H, D) hold the rotated K and the V of every shard, slot t
    (rows [t*S_loc, (t+1)*S_loc)) the shard of rank block_order(rank, W)[t].
    `trace` (a list) collects device events at the schedule's milestones.
    With `check_status` (and W > 1, outside a CUDA-graph capture) the call ends by
    synchronising and raising FaError if the barrier's bounded wait expired;
    a caller that passes False checks `ex.check()` at a point of its own."""
    B, S, H, D = q.shape
    W, r = ex.world, ex.rank
    dev = q.device
    cur = torch.cuda.current_stream(dev)
    par = ex.n_fwd % 2
    ex.n_fwd += 1
    pub_k, pub_v = ex.pub(par)
    _mark(trace, "start")
    if pos is not None:
        q_r = kern.rope(q, pos)
        kern.rope(k, pos, out=pub_k)
    else:
        q_r = q.contiguous()
        pub_k.copy_(k)
    pub_v.copy_(v)
    k_all = torch.empty((B, W * S, H, D), device=dev, dtype=q.dtype)
    v_all = torch.empty_like(k_all)
    # this rank's own shard into slot 0 while every SM is still free
    k_all[:, :S].copy_(pub_k)
    v_all[:, :S].copy_(pub_v)
    o = torch.empty((B, S, H, D), device=dev, dtype=q.dtype)
    lse = torch.empty((B, H, S), device=dev, dtype=torch.float32)
    _mark(trace, "rope+pub")
    if W == 1:
        kern.fwd_fold(q_r, pub_k, pub_v, scale, o, lse, 0, True, o, lse)
        _mark(trace, "fold0.end")
        return o, lse, q_r, k_all, v_all
    ex.barrier(0)  # every rank's shard is published
    _mark(trace, "barrier0")
    # copy engine: the remote shards in fold order
    order = block_order(r, W)
    cs = ex.copy_stream
    cs.wait_stream(cur)
    landed = [None] * W
    for t in range(1, W):
        ex.pull(par, order[t], t, 0, k_all, cs)
        ex.pull(par, order[t], t, 1, v_all, cs)
        _mark(trace, f"pull{t}", cs)  # (before `landed`, which the folds join)
        landed[t] = torch.cuda.Event()
        landed[t].record(cs)
    # two fp32 (O, LSE) accumulators folded on two streams, then merged
    acc = [(torch.empty((B, S, H, D), device=dev, dtype=torch.float32),
            torch.empty((B, H, S), device=dev, dtype=torch.float32)) for _ in range(2)]
    side = ex.side_stream
    side.wait_stream(cur)
    steps = [0, 0]
    for g, slots in enumerate(fold_groups(W)):
        a = g % 2
        st = cur if a == 0 else side
        for t in slots:
            if landed[t] is not None:
                st.wait_event(landed[t])
        lo, hi = slots[0] * S, (slots[-1] + 1) * S
        kb, vb = (pub_k, pub_v) if slots == [0] else (k_all[:, lo:hi], v_all[:, lo:hi])
        _mark(trace, f"fold{g}.begin", st)
        kern.fwd_fold(q_r, kb, vb, scale, acc[a][0], acc[a][1], steps[a], False, o, lse,
                      stream=st)
        _mark(trace, f"fold{g}.end", st)
        steps[a] += 1
    cur.wait_stream(side)
    kern.merge(acc[0][0], acc[0][1], acc[1][0], acc[1][1], o, lse)
    _mark(trace, "merge")
    if check_status and not _capturing():
        ex.check()
    return o, lse, q_r, k_all, v_all


def peer_bwd(q_r, k_all, v_all, o, d_o, lse, pos, scale, ex: PeerExchange, kern: PeerKernels,
             trace: Optional[list] = None, check_status: bool = True):
    """(dq, dk, dv) of this rank's rows w.r.t. the pre-rotation q/k.
    `check_status` as in peer_fwd (the backward's barrier)."""
    B, S, H, D = q_r.shape
    W = ex.world
    dev = q_r.device
    par = ex.n_bwd % 2
    ex.n_bwd += 1
    sp = (S + 127) // 128 * 128
    lse2_pad = torch.empty((B, H, sp), device=dev, dtype=torch.float32)
    delta_pad = torch.empty((B, H, sp), device=dev, dtype=torch.float32)
    kern.bwd_prepare(o, d_o, lse, lse2_pad, delta_pad)
    dq_acc = torch.zeros((B, H, sp, D), device=dev, dtype=torch.float32)
    _mark(trace, "prepare")
    # key slot t of k_all belongs to rank block_order(rank, W)[t]
    order = block_order(ex.rank, W)
    dk_ptrs, dv_ptrs = ex.recv_ptrs(par, 0), ex.recv_ptrs(par, 1)
    kern.bwd_scatter(q_r, k_all, v_all, d_o, lse2_pad, delta_pad, dq_acc, S,
                     [dk_ptrs[owner] for owner in order], [dv_ptrs[owner] for owner in order],
                     scale)
    _mark(trace, "scatter")
    if W > 1:
        ex.barrier(1)  # every rank's contribution to this rank's keys has landed
    _mark(trace, "barrier1")
    dq = torch.empty((B, S, H, D), device=dev, dtype=q_r.dtype)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    kern.reduce_cast(ex.recv(par), pos, dk, dv)
    _mark(trace, "reduce")
    kern.cast(dq_acc, 1, scale, pos, dq)
    _mark(trace, "dqcast")
    if check_status and W > 1 and not _capturing():
        ex.check()
    return dq, dk, dv


class _PeerAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, pos, scale, ex, kern):
        o, lse, q_r, k_all, v_all = peer_fwd(q, k, v, pos, scale, ex, kern)
        ctx.save_for_backward(q_r, k_all, v_all, o, lse)
        ctx.pos, ctx.scale, ctx.ex, ctx.kern = pos, scale, ex, kern
        return o

    @staticmethod
    def backward(ctx, grad_o):
        q_r, k_all, v_all, o, lse = ctx.saved_tensors
        dq, dk, dv = peer_bwd(q_r, k_all, v_all, o, grad_o.contiguous(), lse, ctx.pos, ctx.scale,
                              ctx.ex, ctx.kern)
        return dq, dk, dv, None, None, None, None


def peer_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, ex: PeerExchange,
                   pos: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                   kernels: Optional[PeerKernels] = None) -> torch.Tensor:
    """Attention of this rank's rows (B, S_loc, H, D) against the whole
    sequence sharded over `ex`'s ranks; differentiable. `pos` are this
    shard's (S_loc, 4) axial positions (RoPE applied inside), or None."""
    q4, k4, v4 = ops.as_bshd(q), ops.as_bshd(k), ops.as_bshd(v)
    if k4.shape != q4.shape or v4.shape != q4.shape:
        raise ValueError("q, k, v shards must share one shape")
    if tuple(q4.shape) != ex.shape:
        raise ValueError(f"shard shape {tuple(q4.shape)} != the exchange's {ex.shape}")
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise TypeError("the peer path computes in bf16")
    kern = kernels if kernels is not None else PeerKernels()
    scale = ops.default_scale(q4.shape[-1]) if scale is None else float(scale)
    o = _PeerAttention.apply(q4, k4, v4, pos, scale, ex, kern)
    return o if q.dim() == 4 else o.squeeze(0)
