"""Test support for the peer-memory sequence-parallel path
(`foundry_trainer_b200.peer`).

TEST INFRASTRUCTURE ONLY.

`ThreadPeers(W)` stands W ranks up as W threads of one process on one GPU:
`exchange(rank)` returns an object with PeerExchange's surface whose
published shards and receive slots are ordinary device tensors of that one
GPU, whose pulls are the same `fa_copy_2d` copies (device-local here), and
whose barrier is a device synchronise followed by a host thread barrier — no
kernel waits on another, so the ranks' kernels only ever run side by side.
The real schedule (`peer_fwd` / `peer_bwd`, the C ABI kernels, the scatter
of dK/dV rows into the owners' slots) runs unchanged on top of it.

`peer_rank` is one process of the real thing: one GPU per rank, the IPC
buffers, copy-engine pulls and the device barrier (`PeerExchange`).
"""
from __future__ import annotations

import os
import threading
from datetime import timedelta

import torch


class ThreadPeers:
    def __init__(self, world: int, shape, device="cuda", copy="ce"):
        self.world = world
        self.copy = copy
        self.shape = tuple(shape)
        self.barrier_ = threading.Barrier(world, timeout=120)
        B, S, H, D = self.shape
        self.pub = [[[torch.zeros(self.shape, device=device, dtype=torch.bfloat16)
                      for _ in range(2)] for _ in range(2)] for _ in range(world)]
        self.recv = [[torch.zeros((world, 2) + self.shape, device=device, dtype=torch.float32)
                      for _ in range(2)] for _ in range(world)]

    def exchange(self, rank: int):
        peers = self

        class _Exchange:
            world = peers.world
            shape = peers.shape

            def __init__(self):
                self.rank = rank
                self.copy_stream = torch.cuda.Stream()
                self.side_stream = torch.cuda.Stream()
                self.n_fwd = 0
                self.n_bwd = 0

            def pub(self, par):
                return tuple(peers.pub[rank][par])

            def recv(self, par):
                return peers.recv[rank][par]

            def recv_ptrs(self, par, which):
                return [peers.recv[o][par][rank, which].data_ptr() for o in range(peers.world)]

            def barrier(self, channel, stream=None):
                torch.cuda.synchronize()
                peers.barrier_.wait()

            def check(self):
                from foundry_trainer_b200 import _lib, ops
                _lib.check(ops.device_status(), "thread peers")

            def pull(self, par, src, slot, which, dst, stream):
                from foundry_trainer_b200 import _lib, ops
                B, S, H, D = peers.shape
                row = S * H * D * 2
                src_ptr = peers.pub[src][par][which].data_ptr()
                lib = _lib.load()
                args = (dst.data_ptr() + slot * row, peers.world * row, src_ptr, row, row, B)
                if peers.copy == "sm":
                    rc = lib.fa_copy_2d_sm(*args, 148, ops._stream_ptr(stream))
                else:
                    rc = lib.fa_copy_2d(*args, ops._stream_ptr(stream))
                assert rc == 0, rc

        return _Exchange()


def peer_rank(rank, world, port, arrays, results, steps=1, copy="ce"):
    """One process per GPU: peer_attention of its shard, `steps` times (the
    results of the last step are reported)."""
    import torch.distributed as dist

    from foundry_trainer_b200 import ops, peer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    ex = None
    try:
        q, k, v, d_o, pos = (torch.from_numpy(a) for a in arrays)
        n = q.shape[1] // world
        sl = slice(rank * n, (rank + 1) * n)
        B, _, H, D = q.shape
        ex = peer.PeerExchange(B, n, H, D, copy=copy)
        for _ in range(steps):
            to = lambda t: t[:, sl].to(torch.bfloat16).cuda().requires_grad_(True)
            qs, ks, vs = to(q), to(k), to(v)
            o = peer.peer_attention(qs, ks, vs, ex=ex, pos=pos[sl].contiguous().cuda())
            o.backward(d_o[:, sl].to(torch.bfloat16).cuda())
        torch.cuda.synchronize()
        status = ops.device_status()
        f = lambda t: t.detach().float().cpu().numpy()
        results.put((rank, f(o), f(qs.grad), f(ks.grad), f(vs.grad), status))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


# ------------------------------------------------- gloo (CPU) stand-ins
class _NoStream:
    """Stream stand-in for CPU ranks: ordering is program order."""

    def wait_stream(self, other):
        pass

    def wait_event(self, event):
        pass


class _NoEvent:
    def __init__(self, *args, **kwargs):
        pass

    def record(self, stream=None):
        pass


class GlooExchange:
    """PeerExchange's surface for CPU ranks of a gloo group: the published
    shards move by an all-gather at the forward's barrier, the dK/dV rows
    each rank stored for the owners by an all-gather at the backward's
    barrier. The addresses the backward scatters to are (par, owner, src,
    which) handles the stand-in kernels resolve."""

    def __init__(self, shape, dtype=torch.float32):
        import torch.distributed as dist
        self.dist = dist
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.shape = tuple(shape)
        self.copy_stream, self.side_stream = _NoStream(), _NoStream()
        self.n_fwd = self.n_bwd = 0
        self._pub = [[torch.zeros(self.shape, dtype=dtype) for _ in range(2)] for _ in range(2)]
        self._recv = [torch.zeros((self.world, 2) + self.shape) for _ in range(2)]
        self._gathered = [None, None]
        self.outbox = {}
        self.status = 0  # what the device status word would hold

    def pub(self, par):
        return tuple(self._pub[par])

    def recv(self, par):
        return self._recv[par]

    def recv_ptrs(self, par, which):
        return [(par, owner, self.rank, which) for owner in range(self.world)]

    def barrier(self, channel, stream=None):
        """The device barrier's stand-in. Like the device kernel, a barrier
        that cannot complete (a peer left: the gloo collective fails or runs
        into the group's timeout) records FA_ERR_DEVICE_TIMEOUT and returns;
        the data a missing peer would have delivered stays stale (zeros),
        and `check()` raises."""
        dist, W = self.dist, self.world
        if channel == 0:
            par = (self.n_fwd - 1) % 2
            mine = torch.stack(self._pub[par])
            got = [torch.empty_like(mine) for _ in range(W)]
            try:
                dist.all_gather(got, mine)
                dist.barrier()
            except RuntimeError:
                self.status = 5  # FA_ERR_DEVICE_TIMEOUT
                got = [mine if r == self.rank else torch.zeros_like(mine) for r in range(W)]
            self._gathered[par] = got
        else:
            par = (self.n_bwd - 1) % 2
            mine = torch.stack([torch.stack([self.outbox[(par, o, self.rank, w)] for w in (0, 1)])
                                for o in range(W)])  # (owner, which, B, S, H, D)
            got = [torch.empty_like(mine) for _ in range(W)]
            try:
                dist.all_gather(got, mine)
                dist.barrier()
            except RuntimeError:
                self.status = 5
                return
            for src in range(W):
                self._recv[par][src] = got[src][self.rank]

    def check(self):
        from foundry_trainer_b200 import _lib
        status, self.status = self.status, 0
        _lib.check(status, "gloo peers")

    def pull(self, par, src, slot, which, dst, stream):
        S = self.shape[1]
        dst[:, slot * S:(slot + 1) * S].copy_(self._gathered[par][src][which])


def fake_peer_kernels(ex):
    from tests.ring_support import FakeRingKernels, _rope_np

    class FakePeerKernels(FakeRingKernels):
        """peer.PeerKernels' surface on CPU tensors, float64 arithmetic, in
        the conventions of the C ABI calls (fa_fwd_fold, fa_merge_f32,
        fa_bwd_scatter, fa_reduce_cast_f32)."""

        def fwd_fold(self, q, k, v, scale, o_acc, lse_acc, step, last, o, lse, stream=None):
            super().fwd_fold(q, k, v, scale, o_acc, lse_acc, step, last, o, lse)

        def merge(self, o_a, lse_a, o_b, lse_b, o, lse):
            self.calls.append("merge")
            a, b = lse_a.double(), lse_b.double()
            m = torch.maximum(a, b)
            wa, wb = torch.exp(a - m), torch.exp(b - m)
            tr = lambda x: x.permute(0, 2, 1)[..., None]
            o.copy_((o_a.double() * tr(wa) + o_b.double() * tr(wb)) / tr(wa + wb))
            lse.copy_(m + torch.log(wa + wb))

        def bwd_scatter(self, q, k_all, v_all, d_o, lse2_pad, delta_pad, dq_acc, seg,
                        dk_ptrs, dv_ptrs, scale):
            B, S, H, D = q.shape
            kv = k_all.shape[1]
            dk = torch.empty((B, kv, H, D))
            dv = torch.empty((B, kv, H, D))
            self.bwd_partial(q, k_all, v_all, d_o, lse2_pad, delta_pad, dq_acc, dk, dv, scale,
                             False)
            for i, (hk, hv) in enumerate(zip(dk_ptrs, dv_ptrs)):
                ex.outbox[hk] = dk[:, i * seg:(i + 1) * seg].clone()
                ex.outbox[hv] = dv[:, i * seg:(i + 1) * seg].clone()

        def reduce_cast(self, recv, pos, dk, dv):
            self.calls.append("reduce_cast")
            sk = recv[:, 0].double().sum(0)
            if pos is not None:
                sk = _rope_np(sk.float(), pos, inverse=True).double()
            dk.copy_(sk)
            dv.copy_(recv[:, 1].double().sum(0))

    return FakePeerKernels()


def peer_gloo_rank(rank, world, port, shape, seed, results, steps=2):
    """One gloo rank: the peer-memory schedule (peer.peer_fwd / peer_bwd) of
    its shard with the CPU stand-ins; the last step's results are reported."""
    import torch.distributed as dist

    from foundry_trainer_b200 import ops, peer
    from tests.ring_support import full_problem

    torch.cuda.current_stream = lambda *a, **k: _NoStream()
    torch.cuda.Event = _NoEvent
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        B, S, H, D = shape
        q, k, v, d_o, pos = full_problem(B, S, H, D, seed)
        n = S // world
        sl = slice(rank * n, (rank + 1) * n)
        qs, ks, vs, dos = (t[:, sl].contiguous() for t in (q, k, v, d_o))
        ps = pos[sl].contiguous()
        ex = GlooExchange((B, n, H, D))
        kern = fake_peer_kernels(ex)
        scale = ops.default_scale(D)
        for _ in range(steps):
            o, lse, q_r, k_all, v_all = peer.peer_fwd(qs, ks, vs, ps, scale, ex, kern)
            dq, dk, dv = peer.peer_bwd(q_r, k_all, v_all, o, dos, lse, ps, scale, ex, kern)
        results.put((rank, o.numpy(), dq.numpy(), dk.numpy(), dv.numpy(), kern.calls))
    finally:
        dist.destroy_process_group()


def peer_gloo_rank_leaves(rank, world, port, shape, seed, results, leave_after=1,
                          timeout_s=10.0):
    """Failure detection on gloo ranks: every rank runs the peer schedule;
    the last rank leaves after `leave_after` fwd+bwd steps (between steps,
    nothing of its own in flight), the others go on to the next step. A
    survivor's barrier cannot complete, records the timeout status, and the
    step's status check raises FaError instead of hanging. Reports (rank,
    steps completed, status code of the raised error or 0, seconds)."""
    import time

    import torch.distributed as dist

    from foundry_trainer_b200 import _lib, ops, peer
    from tests.ring_support import full_problem

    torch.cuda.current_stream = lambda *a, **k: _NoStream()
    torch.cuda.Event = _NoEvent
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    done, code, t0 = 0, 0, time.time()
    try:
        B, S, H, D = shape
        q, k, v, d_o, pos = full_problem(B, S, H, D, seed)
        n = S // world
        sl = slice(rank * n, (rank + 1) * n)
        qs, ks, vs, dos = (t[:, sl].contiguous() for t in (q, k, v, d_o))
        ps = pos[sl].contiguous()
        ex = GlooExchange((B, n, H, D))
        kern = fake_peer_kernels(ex)
        scale = ops.default_scale(D)
        steps = leave_after if rank == world - 1 else leave_after + 1
        try:
            for _ in range(steps):
                o, lse, q_r, k_all, v_all = peer.peer_fwd(qs, ks, vs, ps, scale, ex, kern)
                peer.peer_bwd(q_r, k_all, v_all, o, dos, lse, ps, scale, ex, kern)
                done += 1
        except _lib.FaError as e:
            code = e.status
        results.put((rank, done, code, time.time() - t0))
    finally:
        dist.destroy_process_group()
