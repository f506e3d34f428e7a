"""Head-parallel attention: the all-to-all schedule on gloo CPU ranks.

foundry_trainer_b200/heads.py is run by 2 and 3 processes over gloo with the
oracle standing in for the kernels (tests/heads_support.py); the gathered
sequence shards of O, dQ, dK, dV must equal the oracle's single-sequence
result with RoPE at the whole sequence's axial positions. This checks the
two layout exchanges (sequence shards <-> head groups) and the autograd
wiring; the kernels are the single-GPU op, checked on the GPU.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc

TOL = 1e-6  # the stand-in is the oracle itself: only the layouts can differ


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, shape, seed):
    from tests import heads_support
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=heads_support.gloo_rank,
                         args=(r, world, port, shape, seed, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, *vals = results.get(timeout=240)
            got[r] = vals
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [got[r] for r in range(world)]


@pytest.mark.parametrize("world,S,H", [(2, 96, 4), (3, 105, 6)])
def test_head_parallel_matches_single_sequence_oracle(world, S, H):
    from tests import ring_support
    B, D = 1, 128
    q, k, v, d_o, pos = ring_support.full_problem(B, S, H, D, seed=40 + world)
    ref = orc.attn_fwd_bwd_bshd(q.numpy(), k.numpy(), v.numpy(), d_o.numpy(), "f32",
                                rope_pos=pos.numpy())
    shards = _run(world, (B, S, H, D), seed=40 + world)
    for i, name in enumerate(("o", "dq", "dk", "dv")):
        ours = np.concatenate([s[i] for s in shards], axis=1)
        err = orc.max_rel(ours, ref[{"o": 0, "dq": 2, "dk": 3, "dv": 4}[name]])
        assert err <= TOL, (name, err)
    # each rank ran the op once forward and once backward, on its H/W heads
    # over the whole sequence
    for s in shards:
        assert s[4] == [("fwd", (B, S, H // world, D)), ("bwd", (B, S, H // world, D))]


def test_layout_exchange_round_trip_single_rank():
    """W = 1: the exchanges are identities (the op then runs on all heads)."""
    from foundry_trainer_b200 import heads
    ex = heads.HeadExchange()
    x = torch.randn(2, 10, 6, 8)
    (y,) = heads.seq_to_heads([x], ex)
    assert torch.equal(y, x)
    (z,) = heads.heads_to_seq([y], ex)
    assert torch.equal(z, x)


def test_heads_must_divide_over_ranks():
    from foundry_trainer_b200 import heads

    class Three:
        world, rank = 4, 0

        def all_to_all(self, recv, send):
            recv.copy_(send)

    with pytest.raises(ValueError):
        heads.seq_to_heads([torch.zeros(1, 8, 6, 8)], Three())
