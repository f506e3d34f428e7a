"""Head-parallel attention on the GPU (foundry_trainer_b200/heads.py).

* One rank (W = 1): the schedule is the single-GPU op on all heads; against
  the fp32 oracle at the bf16 bound.
* Two processes on two GPUs with NCCL all-to-alls and the real kernels, two
  steps: the gathered shards of O, dQ, dK, dV against the oracle on the
  whole sequence (RoPE at its axial positions), max-rel <= 2e-2 per tensor.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests.helpers import assert_close, np32

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _problem(S, H, seed):
    from tests import ring_support
    q, k, v, d_o, pos = ring_support.full_problem(1, S, H, 128, seed)
    # the bf16-rounded inputs both sides see
    q, k, v, d_o = (t.to(torch.bfloat16).float() for t in (q, k, v, d_o))
    return q, k, v, d_o, pos


def _oracle(q, k, v, d_o, pos):
    return orc.attn_fwd_bwd_bshd(q.numpy(), k.numpy(), v.numpy(), d_o.numpy(), "f32",
                                 rope_pos=pos.numpy())


def test_head_parallel_single_rank_matches_oracle():
    from foundry_trainer_b200 import heads, ops
    q, k, v, d_o, pos = _problem(700, 3, seed=61)
    dev = lambda t: t.to(torch.bfloat16).cuda()
    ex, kern = heads.HeadExchange(), heads.HeadKernels()
    scale = ops.default_scale(128)
    o, state = heads.head_fwd(dev(q), dev(k), dev(v), pos.cuda(), scale, ex, kern)
    dq, dk, dv = heads.head_bwd(dev(d_o), state, scale, ex, kern)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ro, _, rdq, rdk, rdv = _oracle(q, k, v, d_o, pos)
    assert_close({"o": np32(o), "dq": np32(dq), "dk": np32(dk), "dv": np32(dv)},
                 {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "heads w1")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_parallel_two_gpu_ranks_match_oracle():
    from tests import heads_support
    q, k, v, d_o, pos = _problem(2 * 528, 4, seed=62)
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    arrays = tuple(t.numpy() for t in (q, k, v, d_o, pos))
    port = _free_port()
    procs = [ctx.Process(target=heads_support.nccl_rank, args=(r, 2, port, arrays, results, 2))
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
    cat = {n: np.concatenate([got[r][i] for r in range(2)], axis=1)
           for i, n in enumerate(("o", "dq", "dk", "dv"))}
    ro, _, rdq, rdk, rdv = _oracle(q, k, v, d_o, pos)
    assert_close(cat, {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "heads w2")
