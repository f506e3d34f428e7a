"""Ring (sequence-parallel) attention: the host schedule on gloo CPU ranks.

The ring driver (foundry_trainer_b200/ring.py) is run by 2 and 3 processes
over gloo with the CPU stand-in kernels of tests/ring_support.py; the gathered
shards of O, dQ, dK, dV must equal the oracle's single-sequence result (with
RoPE at the shards' axial positions). This checks the exchange order, the
merge and the travelling dK/dV accumulators; the block kernels themselves are
checked against the oracle on the GPU.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

from oracle import attn_oracle as orc

TOL = 1e-4  # f32 path tolerance (the stand-in computes in f64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, shape, seed):
    from tests import ring_support
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=ring_support.gloo_rank, args=(r, world, port, shape, seed, results))
             for r in range(world)]
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


@pytest.mark.parametrize("world,S", [(2, 96), (3, 105)])
def test_ring_matches_single_sequence_oracle(world, S):
    from tests import ring_support
    B, H, D = 1, 2, 128
    q, k, v, d_o, pos = ring_support.full_problem(B, S, H, D, seed=world)
    o_ref, _, dq_ref, dk_ref, dv_ref = orc.attn_fwd_bwd_bshd(
        q.numpy(), k.numpy(), v.numpy(), d_o.numpy(), "f32", rope_pos=pos.numpy())
    shards = _run(world, (B, S, H, D), seed=world)
    cat = lambda i: np.concatenate([s[i] for s in shards], axis=1)
    for name, ours, ref in (("o", cat(0), o_ref), ("dq", cat(1), dq_ref), ("dk", cat(2), dk_ref),
                            ("dv", cat(3), dv_ref)):
        err = orc.max_rel(ours, ref)
        assert err <= TOL, (name, err)
    # every rank ran W forward blocks, W backward blocks and W-1 accumulator adds
    for calls in (s[4] for s in shards):
        assert calls.count("fwd_partial") == world
        assert calls.count("bwd_partial") == world
        assert calls.count("add") == world - 1


def test_peer_schedule_covers_every_shard_once():
    from foundry_trainer_b200 import peer
    for world in range(1, 9):
        for rank in range(world):
            order = peer.block_order(rank, world)
            assert order[0] == rank and sorted(order) == list(range(world))
        groups = peer.fold_groups(world)
        assert groups[0] == [0]
        assert [t for g in groups for t in g] == list(range(world))
        assert all(len(g) <= 2 and g == list(range(g[0], g[-1] + 1)) for g in groups)


def test_peer_layout_regions_are_disjoint_and_aligned():
    from foundry_trainer_b200 import peer
    for world in (1, 2, 8):
        lay = peer.Layout(1, 2112, 24, 128, world, 256)
        spans = [(0, 256)]
        for par in range(2):
            for w in range(2):
                spans.append((lay.pub_off(par, w), lay.pub_off(par, w) + lay.n * 2))
            for src in range(world):
                for w in range(2):
                    o = lay.recv_off(par, src, w)
                    spans.append((o, o + lay.n * 4))
        spans.sort()
        assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
        assert spans[-1][1] <= lay.total
        assert all(a % 16 == 0 for a, _ in spans)


def _run_peer(world, shape, seed):
    from tests import peer_support
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=peer_support.peer_gloo_rank,
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


@pytest.mark.parametrize("world,S", [(2, 96), (3, 105)])
def test_peer_schedule_matches_single_sequence_oracle(world, S):
    # the peer-memory schedule (foundry_trainer_b200/peer.py: fold order and
    # groups, the two accumulators and their merge, the backward's scatter to
    # the owners and their sums) on gloo ranks with CPU stand-ins for the
    # device calls and the exchange
    from tests import ring_support
    B, H, D = 1, 2, 128
    q, k, v, d_o, pos = ring_support.full_problem(B, S, H, D, seed=10 + world)
    o_ref, _, dq_ref, dk_ref, dv_ref = orc.attn_fwd_bwd_bshd(
        q.numpy(), k.numpy(), v.numpy(), d_o.numpy(), "f32", rope_pos=pos.numpy())
    shards = _run_peer(world, (B, S, H, D), seed=10 + world)
    cat = lambda i: np.concatenate([s[i] for s in shards], axis=1)
    for name, ours, ref in (("o", cat(0), o_ref), ("dq", cat(1), dq_ref), ("dk", cat(2), dk_ref),
                            ("dv", cat(3), dv_ref)):
        assert orc.max_rel(ours, ref) <= TOL, (name, orc.max_rel(ours, ref))
    calls = shards[0][4]
    assert calls.count("merge") == 2 and calls.count("reduce_cast") == 2  # two steps


@pytest.mark.parametrize("world", [2, 3])
def test_peer_schedule_survivors_raise_timeout_when_a_rank_leaves(world):
    # failure detection (no GPU): the last rank leaves between steps; the
    # survivors' next barrier cannot complete, records FA_ERR_DEVICE_TIMEOUT
    # like the device barrier's bounded wait, and peer_fwd's status check
    # raises instead of the step returning wrong results or hanging
    from tests import peer_support
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    shape = (1, 24 * world, 2, 128)
    procs = [ctx.Process(target=peer_support.peer_gloo_rank_leaves,
                         args=(r, world, port, shape, 3, results, 1, 10.0))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, done, code, secs = results.get(timeout=120)
            got[r] = (done, code, secs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert got[world - 1][:2] == (1, 0)  # the leaver finished its one step cleanly
    for r in range(world - 1):
        done, code, secs = got[r]
        assert done == 1 and code == 5, (r, got[r])  # FA_ERR_DEVICE_TIMEOUT on step 2
        assert secs < 90, (r, secs)
