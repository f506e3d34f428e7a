"""Failure detection on one GPU without a fault: bounded device waits run out.

The peer exchange's barrier kernel (csrc/peer.cu) waits on flags that other
GPUs write, bounded in wall time. Here it runs as rank 0 of 2 with a second,
local flag block standing in for rank 1, which never arrives: nothing sets
the flag it waits on, the wait gives up after 50 ms, the kernel records
FA_ERR_DEVICE_TIMEOUT in the device status word and returns. Only that one
kernel waits; no kernel waits on another. The tests check the status, that
the peer schedule's own status check turns it into an error, and that the
context is still usable (a normal forward + backward afterwards matches the
oracle).
"""
import ctypes as C
import time

import pytest
import torch

from oracle import attn_oracle as orc
from tests.helpers import assert_close, np32

pytestmark = pytest.mark.gpu

TIMEOUT_S = 0.05


def _flag_blocks(n=2):
    from foundry_trainer_b200 import _lib
    words = (int(_lib.load().fa_peer_flags_bytes()) + 3) // 4
    blocks = [torch.zeros(words, dtype=torch.int32, device="cuda") for _ in range(n)]
    return blocks, (C.c_void_p * n)(*[b.data_ptr() for b in blocks])


def _context_still_usable():
    """A normal forward + backward after the expiry, against the oracle."""
    from tests.helpers import run_op
    g = torch.Generator().manual_seed(9)
    q, k, v = ((torch.randn(1, 200, 2, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
               for _ in range(3))
    d_o = torch.randn(1, 200, 2, 128, generator=g).to(torch.bfloat16).cuda()
    o, lse, dq, dk, dv = run_op(q, k, v, d_o)  # asserts a clean status word
    ro, rlse, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "f32")
    assert_close({"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv},
                 {"o": ro, "lse": rlse, "dq": rdq, "dk": rdk, "dv": rdv}, 2e-2, "after expiry")


def test_peer_barrier_wait_expires_with_timeout_status():
    from foundry_trainer_b200 import _lib, ops
    lib = _lib.load()
    assert ops.device_status() == 0
    blocks, flags = _flag_blocks()
    t0 = time.perf_counter()
    rc = lib.fa_peer_barrier(0, 2, flags, 0, TIMEOUT_S, ops._stream_ptr(None))
    assert rc == _lib.FA_OK
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed >= TIMEOUT_S * 0.9, elapsed  # it waited ...
    assert elapsed < 5.0, elapsed               # ... and gave up
    assert ops.device_status() == _lib.FA_ERR_DEVICE_TIMEOUT
    assert ops.device_status() == 0  # read and cleared
    # rank 0 announced itself to "rank 1" (channel 0, source slot 0) before waiting
    assert int(blocks[1][0].item()) == 1
    _context_still_usable()


class _LoneRank:
    """PeerExchange's surface for rank 0 of 2 on one GPU, whose peer never
    arrives: the barrier is the real bounded device barrier over a local
    stand-in flag block for the peer; the absent peer's shard (pulled after
    the barrier) and its receive slots are local buffers nobody fills."""

    world, rank = 2, 0

    def __init__(self, shape):
        from foundry_trainer_b200 import peer
        self.shape = tuple(shape)
        bf, f32 = torch.bfloat16, torch.float32
        self._pub = [[torch.zeros(shape, device="cuda", dtype=bf) for _ in range(2)]
                     for _ in range(2)]
        self._recv = [torch.zeros((2, 2) + self.shape, device="cuda", dtype=f32) for _ in range(2)]
        self._peer_pub = torch.zeros(shape, device="cuda", dtype=bf)
        self._peer_recv = torch.zeros((2, 2) + self.shape, device="cuda", dtype=f32)
        self._blocks, self._flags = _flag_blocks()
        self.copy_stream, self.side_stream = torch.cuda.Stream(), torch.cuda.Stream()
        self.n_fwd = self.n_bwd = 0
        self.check = lambda: peer.PeerExchange.check(self)  # the product's status check

    def pub(self, par):
        return tuple(self._pub[par])

    def recv(self, par):
        return self._recv[par]

    def recv_ptrs(self, par, which):
        return [self._recv[par][0, which].data_ptr(), self._peer_recv[par, which].data_ptr()]

    def barrier(self, channel, stream=None):
        from foundry_trainer_b200 import _lib, ops
        _lib.check(_lib.load().fa_peer_barrier(0, 2, self._flags, channel, TIMEOUT_S,
                                               ops._stream_ptr(stream)), "fa_peer_barrier")

    def pull(self, par, src, slot, which, dst, stream):
        S = self.shape[1]
        with torch.cuda.stream(stream):
            dst[:, slot * S:(slot + 1) * S].copy_(self._peer_pub)


def test_peer_schedule_raises_when_a_peer_never_arrives():
    from foundry_trainer_b200 import _lib, ops, peer
    from tests import ring_support
    B, S, H = 1, 256, 2
    q, k, v, d_o, pos = ring_support.full_problem(B, 2 * S, H, 128, 4)
    qs, ks, vs, dos = (t[:, :S].to(torch.bfloat16).cuda() for t in (q, k, v, d_o))
    ps = pos[:S].contiguous().cuda()
    ex, kern = _LoneRank((B, S, H, 128)), peer.PeerKernels()
    scale = ops.default_scale(128)
    with pytest.raises(_lib.FaError) as fwd_err:
        peer.peer_fwd(qs, ks, vs, ps, scale, ex, kern)
    assert fwd_err.value.status == _lib.FA_ERR_DEVICE_TIMEOUT
    # the same forward without the check (as a caller that checks later) returns;
    # the backward's own barrier then runs out and its check raises
    o, lse, q_r, k_all, v_all = peer.peer_fwd(qs, ks, vs, ps, scale, ex, kern,
                                              check_status=False)
    with pytest.raises(_lib.FaError) as bwd_err:
        peer.peer_bwd(q_r, k_all, v_all, o, dos, lse, ps, scale, ex, kern)
    assert bwd_err.value.status == _lib.FA_ERR_DEVICE_TIMEOUT
    assert ops.device_status() == 0
    _context_still_usable()
