"""The peer-memory sequence-parallel path on the GPU
(`foundry_trainer_b200.peer`, csrc/peer.cu, the backward's scatter mode).

* kernels on one GPU: `fa_bwd_scatter` against `fa_bwd_partial` (the same
  rows, split over segments: bit-identical), `fa_merge_f32` of two folded
  halves against the one-pass forward, `fa_reduce_cast_f32` against a
  sequential fp32 sum cast by `fa_cast_f32`;
* one rank (no process group): the whole path with a real PeerExchange
  (IPC allocation, copy-engine copies of its own shard);
* W ranks emulated by threads on one GPU (tests/peer_support.ThreadPeers):
  the real schedule over device-local stand-ins of the peer buffers;
* 2 ranks on 2 GPUs when the box has them: IPC mappings, copy-engine pulls
  from the peer, the device barrier, peer stores of the dK/dV rows.
Each end-to-end case is compared with the fp32 oracle on the whole sequence
(RoPE at the shards' axial positions) at the bf16 tolerance, 2e-2 max-rel.
"""
import multiprocessing as mp
import socket
import threading

import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests import peer_support, ring_support

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


def _cuda_bf16(*ts):
    return tuple(t.to(torch.bfloat16).cuda() for t in ts)


def test_bwd_scatter_matches_partial_rows():
    from foundry_trainer_b200 import ops, peer, ring
    torch.manual_seed(0)
    S, W, H = 300, 3, 2  # ragged 128-row tiles; key tiles straddle segments
    q, d_o = _cuda_bf16(torch.randn(1, S, H, 128) * 0.5, torch.randn(1, S, H, 128))
    k, v = _cuda_bf16(torch.randn(1, W * S, H, 128) * 0.5, torch.randn(1, W * S, H, 128) * 0.5)
    scale = ops.default_scale(128)
    o = torch.empty_like(q)
    lse = torch.empty((1, H, S), device="cuda")
    rk, pk = ring.RingKernels(), peer.PeerKernels()
    pk.fwd_fold(q, k, v, scale, o, lse, 0, True, o, lse)  # one block over all W*S keys
    sp = 384
    lse2 = torch.empty((1, H, sp), device="cuda")
    delta = torch.empty((1, H, sp), device="cuda")
    rk.bwd_prepare(o, d_o, lse, lse2, delta)
    dq_a = torch.zeros((1, H, sp, 128), device="cuda")
    dk_a = torch.empty((1, W * S, H, 128), device="cuda")
    dv_a = torch.empty_like(dk_a)
    rk.bwd_partial(q, k, v, d_o, lse2, delta, dq_a, dk_a, dv_a, scale, False)
    dq_b = torch.zeros_like(dq_a)
    seg_k = [torch.full((1, S, H, 128), float("nan"), device="cuda") for _ in range(W)]
    seg_v = [torch.full((1, S, H, 128), float("nan"), device="cuda") for _ in range(W)]
    pk.bwd_scatter(q, k, v, d_o, lse2, delta, dq_b, S, [t.data_ptr() for t in seg_k],
                   [t.data_ptr() for t in seg_v], scale)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(torch.cat(seg_k, dim=1), dk_a)
    assert torch.equal(torch.cat(seg_v, dim=1), dv_a)
    # dQ is accumulated by reduce-adds in arrival order: equal up to fp32 reassociation
    assert torch.allclose(dq_b, dq_a, rtol=1e-5, atol=1e-5)


def test_merge_of_two_folded_halves_matches_one_pass():
    from foundry_trainer_b200 import ops, peer
    torch.manual_seed(1)
    S, H = 520, 3
    q, k, v = _cuda_bf16(*(torch.randn(1, S, H, 128) * 0.5 for _ in range(3)))
    scale = ops.default_scale(128)
    o_ref = torch.empty_like(q)
    lse_ref = torch.empty((1, H, S), device="cuda")
    ops.attn_fwd(q, k, v, out=o_ref, lse=lse_ref)
    pk = peer.PeerKernels()
    o = torch.empty_like(q)
    lse = torch.empty_like(lse_ref)
    accs = [(torch.empty((1, S, H, 128), device="cuda"), torch.empty((1, H, S), device="cuda"))
            for _ in range(2)]
    halves = [(0, 200), (200, S)]
    for (a, b), (oa, la) in zip(halves, accs):
        pk.fwd_fold(q, k[:, a:b], v[:, a:b], scale, oa, la, 0, False, o, lse)
    pk.merge(accs[0][0], accs[0][1], accs[1][0], accs[1][1], o, lse)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.allclose(lse, lse_ref, rtol=0, atol=2e-5)
    assert orc.max_rel(o.float().cpu().numpy(), o_ref.float().cpu().numpy()) <= 1e-2


def test_reduce_cast_matches_sum_then_cast():
    from foundry_trainer_b200 import peer, ring
    torch.manual_seed(2)
    W, S, H = 5, 130, 3
    recv = torch.randn((W, 2, 1, S, H, 128), device="cuda")
    pos = ring_support.full_problem(1, S, 1, 128, 0)[4].cuda()
    dk = torch.empty((1, S, H, 128), device="cuda", dtype=torch.bfloat16)
    dv = torch.empty_like(dk)
    peer.PeerKernels().reduce_cast(recv, pos, dk, dv)
    acc_k, acc_v = recv[0, 0].clone(), recv[0, 1].clone()
    for p in range(1, W):
        acc_k += recv[p, 0]
        acc_v += recv[p, 1]
    rk = ring.RingKernels()
    ref_k = rk.cast(acc_k, 0, 1.0, pos, torch.empty_like(dk))
    ref_v = rk.cast(acc_v, 0, 1.0, None, torch.empty_like(dv))
    torch.cuda.synchronize()
    assert torch.equal(dv, ref_v)
    d = (dk.float() - ref_k.float()).abs().max().item()
    assert d <= 1e-2 * ref_k.float().abs().max().item(), d


def _shard(t, world, rank):
    n = t.shape[1] // world
    return t[:, rank * n:(rank + 1) * n]


def _run_rank(world, rank, ex, q, k, v, d_o, pos):
    from foundry_trainer_b200 import ops, peer
    qs, ks, vs, dos = _cuda_bf16(*(_shard(t, world, rank) for t in (q, k, v, d_o)))
    n = q.shape[1] // world
    ps = pos[rank * n:(rank + 1) * n].contiguous().cuda()
    kern, scale = peer.PeerKernels(), ops.default_scale(128)
    # the autograd engine runs every CUDA backward of a device on one worker
    # thread, so threads standing in for ranks call the schedule directly
    o, lse, q_r, k_all, v_all = peer.peer_fwd(qs, ks, vs, ps, scale, ex, kern)
    dq, dk, dv = peer.peer_bwd(q_r, k_all, v_all, o, dos, lse, ps, scale, ex, kern)
    torch.cuda.synchronize()
    f = lambda t: t.detach().float().cpu().numpy()
    return f(o), f(dq), f(dk), f(dv)


def test_peer_single_rank_matches_oracle():
    from foundry_trainer_b200 import ops, peer
    q, k, v, d_o, pos = _problem(680, 2, seed=21)
    ex = peer.PeerExchange(1, 680, 2, 128)
    try:
        for _ in range(3):  # both buffer parities, then the first again
            out = _run_rank(1, 0, ex, q, k, v, d_o, pos)
    finally:
        ex.close()
    assert ops.device_status() == 0
    _check([out], _oracle(q, k, v, d_o, pos), "peer w1")


def test_peer_single_rank_autograd():
    from foundry_trainer_b200 import ops, peer
    q, k, v, d_o, pos = _problem(400, 2, seed=22)
    ex = peer.PeerExchange(1, 400, 2, 128)
    try:
        qs, ks, vs = (t.requires_grad_(True) for t in _cuda_bf16(q, k, v))
        o = peer.peer_attention(qs, ks, vs, ex=ex, pos=pos.cuda())
        o.backward(d_o.to(torch.bfloat16).cuda())
        torch.cuda.synchronize()
    finally:
        ex.close()
    assert ops.device_status() == 0
    f = lambda t: t.detach().float().cpu().numpy()
    _check([(f(o), f(qs.grad), f(ks.grad), f(vs.grad))], _oracle(q, k, v, d_o, pos), "autograd")


@pytest.mark.parametrize("world,S,copy", [(2, 512, "ce"), (3, 900, "ce"), (4, 1056, "ce"),
                                          (8, 1024, "ce"), (4, 1056, "sm")])
def test_peer_thread_emulated_ranks_match_oracle(world, S, copy):
    from foundry_trainer_b200 import ops
    q, k, v, d_o, pos = _problem(S, 2, seed=30 + world)
    peers = peer_support.ThreadPeers(world, (1, S // world, 2, 128), copy=copy)
    outs, errors = [None] * world, []

    def body(r):
        try:
            ex = peers.exchange(r)
            for _ in range(2):  # both buffer parities
                outs[r] = _run_rank(world, r, ex, q, k, v, d_o, pos)
        except BaseException as e:  # surfaced below
            errors.append(e)
            peers.barrier_.abort()

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


def test_copy_rows_kernel_matches_strided_copy():
    from foundry_trainer_b200 import _lib, ops
    src = torch.randint(0, 255, (3, 5000 * 16), dtype=torch.uint8, device="cuda")
    dst = torch.zeros((3, 7000 * 16), dtype=torch.uint8, device="cuda")
    rc = _lib.load().fa_copy_2d_sm(dst.data_ptr() + 512, dst.stride(0), src.data_ptr(),
                                   src.stride(0), 4992 * 16, 3, 37, ops._stream_ptr(None))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(dst[:, 512:512 + 4992 * 16], src[:, :4992 * 16])
    assert int(dst[:, :512].sum()) == 0 and int(dst[:, 512 + 4992 * 16:].sum()) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("copy", ["ce", "sm"])
def test_peer_two_gpu_ranks_match_oracle(copy):
    q, k, v, d_o, pos = _problem(2 * 1056, 3, seed=5)
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    arrays = tuple(t.numpy() for t in (q, k, v, d_o, pos))
    port = _free_port()
    procs = [ctx.Process(target=peer_support.peer_rank,
                         args=(r, 2, port, arrays, results, 3, copy)) for r in range(2)]
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
    _check([got[r][:4] for r in range(2)], _oracle(q, k, v, d_o, pos), f"peer w2 {copy}")
