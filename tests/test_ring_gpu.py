"""Ring attention on the GPU: the bf16 block kernels composed by the ring.

* one rank (no process group): the ring reduces to one block per direction;
* W ranks emulated by threads on one GPU (tests/ring_support.ThreadRing):
  every block call of the real schedule — fa_fwd_partial on ragged 128-row
  tiles, fa_lse_merge, fa_bwd_prepare, fa_bwd_partial in store mode,
  fa_add_f32 and the un-rotating fa_cast_f32 — on real K/V shards;
* 2 NCCL ranks on 2 GPUs when the box has them.
Each is compared with the fp32 oracle on the whole sequence, RoPE at the
shards' axial positions, at the bf16 tolerance (2e-2 max-relative).
"""
import multiprocessing as mp
import socket
import threading

import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests import ring_support

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _bf16(t):
    return t.to(torch.bfloat16).float()


def _problem(S, H, seed):
    q, k, v, d_o, pos = ring_support.full_problem(1, S, H, 128, seed)
    return tuple(_bf16(t) for t in (q, k, v, d_o)) + (pos,)


def _oracle(q, k, v, d_o, pos):
    o, _, dq, dk, dv = orc.attn_fwd_bwd_bshd(q.numpy(), k.numpy(), v.numpy(), d_o.numpy(), "f32",
                                             rope_pos=pos.numpy())
    return {"o": o, "dq": dq, "dk": dk, "dv": dv}


def _check(shards, ref, label):
    for i, name in enumerate(("o", "dq", "dk", "dv")):
        ours = np.concatenate([s[i] for s in shards], axis=1)
        err = orc.max_rel(ours, ref[name])
        assert err <= TOL, (label, name, err)


def _rank(world, rank, comm, q, k, v, d_o, pos, autograd=True):
    from foundry_trainer_b200 import ops, ring
    n = q.shape[1] // world
    sl = slice(rank * n, (rank + 1) * n)
    to = lambda t: t[:, sl].to(torch.bfloat16).cuda()
    qs, ks, vs, dos, ps = to(q), to(k), to(v), to(d_o), pos[sl].contiguous().cuda()
    f = lambda t: t.detach().float().cpu().numpy()
    if autograd:
        qs, ks, vs = (t.requires_grad_(True) for t in (qs, ks, vs))
        o = ring.ring_attention(qs, ks, vs, pos=ps, comm=comm)
        o.backward(dos)
        torch.cuda.synchronize()
        return f(o), f(qs.grad), f(ks.grad), f(vs.grad)
    # the autograd engine runs every CUDA backward of a device on one worker
    # thread, so threads standing in for ranks call the ring directly
    kern, scale = ring.RingKernels(), ops.default_scale(128)
    o, lse, q_r, k_r = ring.ring_fwd(qs, ks, vs, ps, scale, comm, kern)
    dq, dk, dv = ring.ring_bwd(q_r, k_r, vs, o, dos, lse, ps, scale, comm, kern)
    torch.cuda.synchronize()
    return f(o), f(dq), f(dk), f(dv)


def test_ring_single_rank_matches_oracle():
    from foundry_trainer_b200 import ops, ring
    q, k, v, d_o, pos = _problem(700, 2, seed=11)
    out = _rank(1, 0, ring.RingComm(), q, k, v, d_o, pos)
    assert ops.device_status() == 0
    _check([out], _oracle(q, k, v, d_o, pos), "w1")


@pytest.mark.parametrize("world,S", [(2, 512), (3, 900), (4, 1000)])
def test_ring_thread_emulated_ranks_match_oracle(world, S):
    from foundry_trainer_b200 import ops
    q, k, v, d_o, pos = _problem(S, 2, seed=world)
    ring_ = ring_support.ThreadRing(world)
    outs, errors = [None] * world, []

    def body(r):
        try:
            outs[r] = _rank(world, r, ring_.comm(r), q, k, v, d_o, pos, autograd=False)
        except BaseException as e:  # surfaced below
            errors.append(e)
            ring_.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    assert ops.device_status() == 0
    _check(outs, _oracle(q, k, v, d_o, pos), f"threads w{world}")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ring_two_nccl_ranks_match_oracle():
    q, k, v, d_o, pos = _problem(2 * 1056, 3, seed=5)
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    arrays = tuple(t.numpy() for t in (q, k, v, d_o, pos))
    port = _free_port()
    procs = [ctx.Process(target=ring_support.nccl_rank, args=(r, 2, port, arrays, results))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, *vals = results.get(timeout=300)
            got[r] = vals
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert all(got[r][4] == 0 for r in range(2))
    _check([got[r][:4] for r in range(2)], _oracle(q, k, v, d_o, pos), "nccl w2")
