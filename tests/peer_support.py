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
