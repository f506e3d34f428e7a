"""Fused QK-RMSNorm + RoPE prologue of the joint block on the GPU.

Against the reference's recorded q/k (post RMSNorm + RoPE, both blocks), the
reference generator's autograd gradients, and the oracle on two-stream inputs
(text and image rows from separate tensors, written into the joint tensor).
bf16 tolerances: forward 1e-2 max-relative (it matches the recorded values
to rounding), backward 2e-2.
"""
import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests.helpers import np32

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _bf16(a):
    return torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).cuda()


def test_prologue_matches_reference_recorded_qk(golden_dir):
    from foundry_trainer_b200 import ops
    g = dict(np.load(golden_dir / "rope_fixture_bf16.npz"))
    for c in sorted({k.rsplit("_", 1)[0] for k in g}):
        x = _bf16(g[f"{c}_h"])[None]
        w = _bf16(g[f"{c}_w"])
        rope = ops.Rope(torch.from_numpy(g[f"{c}_pos"]).cuda())
        y = ops.qk_norm_rope(None, x, None, w, rope)
        torch.cuda.synchronize()
        err = orc.max_rel(np32(y)[0], g[f"{c}_post"])
        assert err <= 1e-2, (c, err)


def test_prologue_backward_matches_reference_autograd(golden_dir):
    from foundry_trainer_b200 import ops
    g = dict(np.load(golden_dir / "qk_norm_rope_fixture_bf16.npz"))
    x, w, dy = _bf16(g["x"])[None], _bf16(g["w"]), _bf16(g["dy"])[None]
    rope = ops.Rope(torch.from_numpy(g["pos"]).cuda())
    y = ops.qk_norm_rope(None, x, None, w, rope)
    _, dx, _, dw = ops.qk_norm_rope_bwd(None, x, None, w, rope, dy)
    torch.cuda.synchronize()
    assert orc.max_rel(np32(y)[0], g["y"]) <= 1e-2
    assert orc.max_rel(np32(dx)[0], g["dx"]) <= 2e-2
    assert orc.max_rel(dw.cpu().numpy(), g["dw"]) <= 2e-2


@pytest.mark.parametrize("B,T,grid,H", [(1, 64, 16, 4), (2, 13, 9, 3), (1, 0, 12, 2), (1, 40, 0, 2)])
def test_prologue_two_streams_match_oracle(B, T, grid, H):
    from foundry_trainer_b200 import configs, ops
    I = grid * grid
    gen = torch.Generator().manual_seed(T * 31 + grid)
    x_t = torch.randn(B, T, H, 128, generator=gen) * 3.0
    x_i = torch.randn(B, I, H, 128, generator=gen) * 3.0
    w_t = 1.0 + 0.1 * torch.randn(128, generator=gen)
    w_i = 1.0 + 0.1 * torch.randn(128, generator=gen)
    dy = torch.randn(B, T + I, H, 128, generator=gen)
    pos = configs.positions(T, grid) if grid > 0 else torch.zeros(T, 4)
    xt, xi, wt, wi, dyb = (t.to(torch.bfloat16) for t in (x_t, x_i, w_t, w_i, dy))
    rope = ops.Rope(pos.cuda())
    y = ops.qk_norm_rope(xt.cuda() if T else None, xi.cuda() if I else None,
                         wt.cuda() if T else None, wi.cuda() if I else None, rope)
    dx_t, dx_i, dw_t, dw_i = ops.qk_norm_rope_bwd(
        xt.cuda() if T else None, xi.cuda() if I else None, wt.cuda() if T else None,
        wi.cuda() if I else None, rope, dyb.cuda())
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    f = lambda t: t.float().numpy()
    for b in range(B):
        refs, dxs = [], []
        for lo, hi, xs, ws, dxg in ((0, T, xt, wt, dx_t), (T, T + I, xi, wi, dx_i)):
            if hi == lo:
                continue
            ref = orc.qk_norm_rope(f(xs[b]), f(ws), EPS, pos[lo:hi].numpy(), "bf16")
            err = orc.max_rel(np32(y)[b, lo:hi], ref)
            assert err <= 1e-2, ("y", lo, err)
            rdx, rdw = orc.qk_norm_rope_grad(f(xs[b]), f(ws), EPS, pos[lo:hi].numpy(),
                                            f(dyb[b, lo:hi]), "bf16")
            assert orc.max_rel(np32(dxg)[b], rdx) <= 2e-2, ("dx", lo)
    # the weight gradients sum over the batch
    for lo, hi, xs, ws, dwg in ((0, T, xt, wt, dw_t), (T, T + I, xi, wi, dw_i)):
        if hi == lo:
            continue
        rdw = sum(orc.qk_norm_rope_grad(f(xs[b]), f(ws), EPS, pos[lo:hi].numpy(),
                                        f(dyb[b, lo:hi]), "bf16")[1] for b in range(B))
        assert orc.max_rel(dwg.cpu().numpy(), rdw) <= 2e-2, ("dw", lo)


def test_joint_attention_matches_oracle_chain():
    """The double block's attention from the two streams' projections
    (norm + RoPE + cat fused, attention, narrow) under autograd, against the
    oracle's composition of the reference ops."""
    from foundry_trainer_b200 import attn, configs
    gen = torch.Generator().manual_seed(5)
    B, T, grid, H = 1, 64, 12, 2
    I = grid * grid
    mk = lambda n: (torch.randn(B, n, H, 128, generator=gen) * 2.0).to(torch.bfloat16)
    q_t, k_t, v_t, q_i, k_i, v_i = mk(T), mk(T), mk(T), mk(I), mk(I), mk(I)
    ws = [(1.0 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16) for _ in range(4)]
    do_t, do_i = mk(T), mk(I)
    pos = configs.positions(T, grid)
    dev = [t.cuda().requires_grad_(True) for t in (q_t, k_t, v_t, q_i, k_i, v_i, *ws)]
    op = attn.JointAttention(pos.cuda())
    o_t, o_i = op(*dev)
    torch.autograd.backward([o_t, o_i], [do_t.cuda(), do_i.cuda()])
    torch.cuda.synchronize()
    f = lambda t: t.float().numpy()
    pn = pos.numpy()
    wq_t, wk_t, wq_i, wk_i = (f(w) for w in ws)
    qj = np.concatenate([orc.qk_norm_rope(f(q_t[0]), wq_t, EPS, pn[:T], "bf16"),
                         orc.qk_norm_rope(f(q_i[0]), wq_i, EPS, pn[T:], "bf16")])
    kj = np.concatenate([orc.qk_norm_rope(f(k_t[0]), wk_t, EPS, pn[:T], "bf16"),
                         orc.qk_norm_rope(f(k_i[0]), wk_i, EPS, pn[T:], "bf16")])
    vj = np.concatenate([f(v_t[0]), f(v_i[0])])
    doj = np.concatenate([f(do_t[0]), f(do_i[0])])
    oj = orc.attn_fwd(qj, kj, vj, "f32")
    dqj, dkj, dvj = orc.attn_bwd(qj, kj, vj, doj, "f32")
    dq_t, dwq_t = orc.qk_norm_rope_grad(f(q_t[0]), wq_t, EPS, pn[:T], dqj[:T], "bf16")
    dq_i, dwq_i = orc.qk_norm_rope_grad(f(q_i[0]), wq_i, EPS, pn[T:], dqj[T:], "bf16")
    dk_t, dwk_t = orc.qk_norm_rope_grad(f(k_t[0]), wk_t, EPS, pn[:T], dkj[:T], "bf16")
    dk_i, dwk_i = orc.qk_norm_rope_grad(f(k_i[0]), wk_i, EPS, pn[T:], dkj[T:], "bf16")
    checks = {"o_t": (o_t, oj[:T]), "o_i": (o_i, oj[T:]),
              "dq_t": (dev[0].grad, dq_t), "dk_t": (dev[1].grad, dk_t), "dv_t": (dev[2].grad, dvj[:T]),
              "dq_i": (dev[3].grad, dq_i), "dk_i": (dev[4].grad, dk_i), "dv_i": (dev[5].grad, dvj[T:]),
              "dwq_t": (dev[6].grad, dwq_t), "dwk_t": (dev[7].grad, dwk_t),
              "dwq_i": (dev[8].grad, dwq_i), "dwk_i": (dev[9].grad, dwk_i)}
    for name, (ours, ref) in checks.items():
        got = np32(ours)
        got = got[0] if got.ndim == 4 else got
        err = orc.max_rel(got, ref)
        assert err <= 3e-2, (name, err)
