"""Parity of the benchmarked paths at the benchmarked sizes.

bench.py times, per configuration:
  * C2 (B1 H24 S4608 = 512 text + 64x64 image, bf16, axial RoPE inside the
    op): ops.attn_fwd keeping its workspace (rotated q, k and the (cos, sin)
    table) and ops.attn_bwd reusing it (fa_bwd_saved);
  * C4 (B8, otherwise C2): the same calls over the whole batch;
  * C5 (B1 H24 S16896 = 512 text + 128x128 image): the sequence-parallel
    schedule (peer.peer_fwd / peer.peer_bwd), one rank holding the whole
    sequence at N=1, S/N rows per rank at N>1.
Each is run here exactly that way on the configuration's own seeded inputs
(foundry_trainer_b200.configs.make_inputs) and compared with the fp32 CPU
oracle on the same bf16-rounded inputs, RoPE at the configuration's axial
positions, at the bf16 bound: max |x - ref| / max |ref| <= 2e-2 per tensor.
The oracle covers a subset of heads (and batch elements) where the whole
problem would take the CPU minutes; the selection is stated per test.
"""
import threading

import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests.helpers import assert_close, np32

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _oracle_fwd_all_heads(q, k, v, pos, b=0, head_chunk=4):
    """fp32 oracle O (S, H, D) and LSE (H, S) of batch element b, every head,
    q/k rotated by the oracle's apply_rope first."""
    cos, sin = orc.rope_tables(pos, "f32")
    qb, kb, vb = (np32(t[b]) for t in (q, k, v))
    H = qb.shape[1]
    o, lse = [], []
    for h0 in range(0, H, head_chunk):
        hs = slice(h0, min(h0 + head_chunk, H))
        oo, ll = orc.attn_fwd(orc.apply_rope(qb[:, hs], cos, sin, "f32"),
                              orc.apply_rope(kb[:, hs], cos, sin, "f32"), vb[:, hs], "f32",
                              return_lse=True)
        o.append(oo)
        lse.append(ll)
    return np.concatenate(o, axis=1), np.concatenate(lse, axis=0)


def test_c2_benchmarked_path_full_size():
    """C2 through the bench's own calls. O and LSE on all 24 heads; dQ, dK,
    dV (w.r.t. the pre-rotation q, k) on heads 0, 11 and 23."""
    from foundry_trainer_b200 import configs, ops
    cfg = configs.CONFIGS["c2"]
    q, k, v, d_o = (t.cuda() for t in configs.make_inputs(cfg))
    pos = configs.positions(cfg.txt, cfg.grid)
    rope = ops.Rope(pos.cuda())
    saved = {}
    o, lse = ops.attn_fwd(q, k, v, rope=rope, saved=saved)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, saved=saved)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ro, rlse = _oracle_fwd_all_heads(q, k, v, pos.numpy())
    assert_close({"o": np32(o[0]), "lse": np32(lse[0])}, {"o": ro, "lse": rlse}, TOL,
                 "c2 fwd, 24 heads")
    heads = [0, 11, 23]
    _, _, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "f32",
                                                heads=heads, rope_pos=pos.numpy())
    sel = lambda x: np32(x[:, :, heads])
    assert_close({"dq": sel(dq), "dk": sel(dk), "dv": sel(dv)},
                 {"dq": rdq, "dk": rdk, "dv": rdv}, TOL, "c2 bwd, heads 0/11/23")


def test_c4_batch_full_size_first_and_last_sequence():
    """C4 (B=8) through the same calls over the whole batch; every output of
    batch elements 0 and 7 on heads 0 and 23 against the oracle (the batch
    index reaches the kernels' TMA coordinates and output strides)."""
    from foundry_trainer_b200 import configs, ops
    cfg = configs.CONFIGS["c4"]
    q, k, v, d_o = (t.cuda() for t in configs.make_inputs(cfg))
    pos = configs.positions(cfg.txt, cfg.grid)
    rope = ops.Rope(pos.cuda())
    saved = {}
    o, lse = ops.attn_fwd(q, k, v, rope=rope, saved=saved)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, saved=saved)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    heads = [0, 23]
    for b in (0, 7):
        one = lambda t: np32(t[b:b + 1])
        ro, rlse, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(one(q), one(k), one(v), one(d_o), "f32",
                                                        heads=heads, rope_pos=pos.numpy())
        sel = lambda x: np32(x[b:b + 1, :, heads])
        assert_close({"o": sel(o), "lse": np32(lse[b:b + 1, heads]), "dq": sel(dq),
                      "dk": sel(dk), "dv": sel(dv)},
                     {"o": ro, "lse": rlse, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, f"c4 b={b}")


# ------------------------------------------------------------------- C5
C5_HEADS = [0]


@pytest.fixture(scope="module")
def c5():
    """C5's inputs and the oracle on head 0 over the whole 16896-row sequence
    (about 6 GB of host memory and half a minute of CPU; shared by the
    tests below)."""
    from foundry_trainer_b200 import configs
    cfg = configs.CONFIGS["c5"]
    q, k, v, d_o = configs.make_inputs(cfg)
    pos = configs.positions(cfg.txt, cfg.grid)
    sub = lambda t: np32(t[:, :, C5_HEADS])
    ref = orc.attn_fwd_bwd_bshd(sub(q), sub(k), sub(v), sub(d_o), "f32", rope_pos=pos.numpy())
    return (q, k, v, d_o, pos), dict(zip(("o", "lse", "dq", "dk", "dv"), ref))


def _run_schedule(ex, q, k, v, d_o, pos):
    """peer_fwd + peer_bwd of one rank's shard (the bench's step), as numpy."""
    from foundry_trainer_b200 import ops, peer
    kern, scale = peer.PeerKernels(), ops.default_scale(128)
    o, lse, q_r, k_all, v_all = peer.peer_fwd(q, k, v, pos, scale, ex, kern)
    dq, dk, dv = peer.peer_bwd(q_r, k_all, v_all, o, d_o, lse, pos, scale, ex, kern)
    torch.cuda.synchronize()
    return tuple(np32(t) for t in (o, dq, dk, dv))


def test_c5_one_rank_full_size(c5):
    """C5 at N=1 as bench.py runs it: one rank, the whole sequence, a real
    PeerExchange (both buffer parities); head 0 against the oracle."""
    from foundry_trainer_b200 import ops, peer
    (q, k, v, d_o, pos), ref = c5
    dev = [t.cuda() for t in (q, k, v, d_o)]
    ex = peer.PeerExchange(*q.shape)
    try:
        for _ in range(2):
            out = _run_schedule(ex, *dev, pos.cuda())
    finally:
        ex.close()
    assert ops.device_status() == 0
    assert_close({n: x[:, :, C5_HEADS] for n, x in zip(("o", "dq", "dk", "dv"), out)},
                 {n: ref[n] for n in ("o", "dq", "dk", "dv")}, TOL, "c5 w1")


def test_c5_eight_thread_emulated_ranks_full_size(c5):
    """C5 sharded 2112 rows per rank over 8 ranks emulated by threads on one
    GPU (tests/peer_support.ThreadPeers: the real schedule and kernels,
    device-local stand-ins for the peer buffers, a host barrier); the
    gathered shards' head 0 against the oracle."""
    from foundry_trainer_b200 import ops
    from tests import peer_support
    (q, k, v, d_o, pos), ref = c5
    W = 8
    n = q.shape[1] // W
    peers = peer_support.ThreadPeers(W, (1, n, q.shape[2], 128))
    outs, errors = [None] * W, []

    def body(r):
        try:
            sl = slice(r * n, (r + 1) * n)
            shard = [t[:, sl].contiguous().cuda() for t in (q, k, v, d_o)]
            outs[r] = _run_schedule(peers.exchange(r), *shard, pos[sl].contiguous().cuda())
        except BaseException as e:  # surfaced below
            errors.append(e)
            peers.barrier_.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(W)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors
    assert ops.device_status() == 0
    cat = {n: np.concatenate([o[i] for o in outs], axis=1)[:, :, C5_HEADS]
           for i, n in enumerate(("o", "dq", "dk", "dv"))}
    assert_close(cat, {n: ref[n] for n in ("o", "dq", "dk", "dv")}, TOL, "c5 w8 threads")


def test_c2_deterministic_backward_full_size():
    """C2 with deterministic=1: three repeats bit-identical; the gradients
    equal the default path's up to the fp32 summation order of dQ (whose
    arrival order the default path does not fix)."""
    from foundry_trainer_b200 import configs, ops
    cfg = configs.CONFIGS["c2"]
    q, k, v, d_o = (t.cuda() for t in configs.make_inputs(cfg))
    rope = ops.Rope(configs.positions(cfg.txt, cfg.grid).cuda())
    o, lse = ops.attn_fwd(q, k, v, rope=rope)
    runs = [ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, deterministic=True) for _ in range(3)]
    ref = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for rep in runs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(runs[0], rep))
    for name, a, b in zip(("dq", "dk", "dv"), runs[0], ref):
        err = orc.max_rel(np32(a), np32(b))
        assert err <= 1e-2, (name, err)
