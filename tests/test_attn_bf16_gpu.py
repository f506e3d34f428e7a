"""bf16 tcgen05 path parity against the oracle.

Tolerance: 2e-2 max-relative error per tensor against the fp32 oracle run on
the same bf16-rounded inputs (the reference's own
bf16-vs-fp32 noise floor for attention grads is 1.12e-2 rel-L2,
tools/fixtures/PROVENANCE.md:52-54). The reference's bf16 fixture replay
uses its acceptance metric, cos >= 0.999 and rel-L2 <= 2e-2 (lib.rs:640-667).
"""
import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc
from tests.helpers import assert_close, np32, run_op

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _oracle_f32(q, k, v, d_o, heads=None, rope_pos=None):
    return orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "f32", heads=heads,
                                 rope_pos=rope_pos)


def test_bf16_fixture_replay(golden_dir):
    g = dict(np.load(golden_dir / "attn_fixture_bf16.npz"))
    for blk in ("double", "single"):
        q, k, v, dout = (torch.from_numpy(g[f"{blk}_{n}"]).to(torch.bfloat16).cuda()
                         for n in ("q", "k", "v", "dout"))
        o, lse, dq, dk, dv = run_op(q, k, v, dout)
        for name, ours, ref in (("o", o, g[f"{blk}_attn"]), ("dq", dq, g[f"{blk}_dq"]),
                                ("dk", dk, g[f"{blk}_dk"]), ("dv", dv, g[f"{blk}_dv"])):
            cos, rel = orc.compare(ours, ref)
            assert cos >= 0.999 and rel <= 2e-2, (blk, name, cos, rel)


def test_c2_parity_subset_of_heads():
    from foundry_trainer_b200 import configs
    cfg = configs.CONFIGS["c2"]
    q, k, v, d_o = (t.cuda() for t in configs.make_inputs(cfg))
    o, lse, dq, dk, dv = run_op(q, k, v, d_o)
    heads = [0, 11, 23]
    ro, rlse, rdq, rdk, rdv = _oracle_f32(q, k, v, d_o, heads=heads)
    sel = lambda x: x[:, :, heads, :]
    errs = assert_close({"o": sel(o), "lse": lse[:, heads], "dq": sel(dq), "dk": sel(dk),
                         "dv": sel(dv)},
                        {"o": ro, "lse": rlse, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "c2")
    print("c2 max-rel", errs)
    for x in (o, dq, dk, dv):
        assert np.isfinite(x).all()


@pytest.mark.parametrize("B,S,H", [(1, 1, 1), (1, 24, 2), (2, 130, 3), (1, 333, 2),
                                   (1, 2112, 2), (3, 256, 1)])
def test_bf16_ragged_shapes(B, S, H):
    g = torch.Generator().manual_seed(S * 7 + H)
    shape = (B, S, H, 128)
    q, k, v = ((torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16).cuda() for _ in range(3))
    d_o = torch.randn(shape, generator=g).to(torch.bfloat16).cuda()
    o, lse, dq, dk, dv = run_op(q, k, v, d_o)
    ro, rlse, rdq, rdk, rdv = _oracle_f32(q, k, v, d_o)
    assert_close({"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv},
                 {"o": ro, "lse": rlse, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, f"{B},{S},{H}")


def test_bf16_strided_views_of_fused_qkv():
    """q/k/v as non-contiguous views into one (B, S, 3, H, D) projection."""
    g = torch.Generator().manual_seed(5)
    B, S, H = 2, 300, 4
    qkv = (torch.randn(B, S, 3, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    assert not q.is_contiguous()
    d_o = torch.randn(B, S, H, 128, generator=g).to(torch.bfloat16).cuda()
    o, lse, dq, dk, dv = run_op(q, k, v, d_o)
    ro, rlse, rdq, rdk, rdv = _oracle_f32(q, k, v, d_o)
    assert_close({"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv},
                 {"o": ro, "lse": rlse, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "strided")


def test_bf16_rope_inside_op():
    from foundry_trainer_b200 import configs, ops
    txt, grid, H = 64, 16, 2
    pos = configs.positions(txt, grid)
    S = pos.shape[0]
    g = torch.Generator().manual_seed(11)
    q, k, v = ((torch.randn(1, S, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
               for _ in range(3))
    d_o = torch.randn(1, S, H, 128, generator=g).to(torch.bfloat16).cuda()
    o, lse, dq, dk, dv = run_op(q, k, v, d_o, rope=ops.Rope(pos.cuda()))
    ro, rlse, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "bf16",
                                                    rope_pos=pos.numpy())
    assert_close({"o": o, "dq": dq, "dk": dk, "dv": dv},
                 {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "rope")


def test_bf16_rope_apply_matches_reference_fixture(golden_dir):
    from foundry_trainer_b200 import ops
    r = dict(np.load(golden_dir / "rope_fixture_bf16.npz"))
    for c in sorted({k.rsplit("_", 1)[0] for k in r}):
        x = torch.from_numpy(r[f"{c}_pre"]).to(torch.bfloat16).cuda()
        y = ops.rope_apply(x, ops.Rope(torch.from_numpy(r[f"{c}_pos"]).cuda()))
        torch.cuda.synchronize()
        assert orc.max_rel(np32(y), r[f"{c}_post"]) <= 1e-2, c


def test_c2_full_size_properties():
    """Size-independent identities on every head at C2 (all 24, not a subset):

    sum_s dV[s] = sum_q dO[q] because each P row sums to one; every O element
    lies within the range of its V column; sum_s dK[s] = 0 because each row
    of dS sums to zero.
    """
    from foundry_trainer_b200 import configs, ops
    cfg = configs.CONFIGS["c2"]
    q, k, v, d_o = (t.cuda() for t in configs.make_inputs(cfg))
    o, lse = ops.attn_fwd(q, k, v)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, d_o, lse)
    torch.cuda.synchronize()
    lhs = dv.float().sum(dim=1)
    rhs = d_o.float().sum(dim=1)
    assert ((lhs - rhs).abs().max() / rhs.abs().max()).item() < 2e-2
    vmax = v.float().amax(dim=1, keepdim=True)
    vmin = v.float().amin(dim=1, keepdim=True)
    of = o.float()
    assert bool(((of <= vmax + 1e-2) & (of >= vmin - 1e-2)).all())
    # sum_k dK = 0 for each query row's softmax gradient: sum over keys of dS is 0
    # => sum_s dK[s] = scale * sum_q (sum_k dS[q,k]) Q[q] = 0
    sk = dk.float().sum(dim=1).abs().max().item()
    assert sk < 2e-2 * dk.float().abs().max().item() * 64


def test_bf16_bwd_saved_reuses_forward_rotation():
    """fa_bwd_saved (the forward's rotated q, k and table) gives fa_bwd's result."""
    from foundry_trainer_b200 import configs, ops
    g = torch.Generator().manual_seed(21)
    txt, grid = 104, 24  # 104 text + 24x24 image tokens
    B, S, H = 1, txt + grid * grid, 3
    q, k, v = ((torch.randn(B, S, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
               for _ in range(3))
    d_o = torch.randn(B, S, H, 128, generator=g).to(torch.bfloat16).cuda()
    pos = configs.positions(txt, grid)
    rope = ops.Rope(pos.cuda())
    saved = {}
    o, lse = ops.attn_fwd(q, k, v, rope=rope, saved=saved)
    assert saved and saved["ws"].numel() > 0
    got = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, saved=saved)
    ref = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for name, a, b in zip(("dq", "dk", "dv"), got, ref):
        # same kernels on the same data; dQ's fp32 reductions may land in another order
        err = orc.max_rel(np32(a), np32(b))
        assert err <= 1e-2, (name, err)
    ro, rlse, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "bf16",
                                                    rope_pos=pos.numpy())
    assert_close({"o": np32(o), "dq": np32(got[0]), "dk": np32(got[1]), "dv": np32(got[2])},
                 {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "bwd_saved")


def test_bf16_op_mirror_with_rope_under_autograd():
    """AttnBwd with RoPE through apply_op3: the backward reuses the forward's rotation."""
    from foundry_trainer_b200 import attn, configs, ops
    g = torch.Generator().manual_seed(23)
    pos = configs.positions(64, 16)
    B, S, H = 1, pos.shape[0], 2
    q, k, v = ((torch.randn(B, S, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
               .requires_grad_(True) for _ in range(3))
    d_o = torch.randn(B, S, H, 128, generator=g).to(torch.bfloat16).cuda()
    op = attn.AttnBwd(rope=ops.Rope(pos.cuda()))
    out = attn.apply_op3(q, k, v, op)
    out.backward(d_o)
    torch.cuda.synchronize()
    ro, _, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "bf16",
                                                 rope_pos=pos.numpy())
    assert_close({"o": np32(out), "dq": np32(q.grad), "dk": np32(k.grad), "dv": np32(v.grad)},
                 {"o": ro, "dq": rdq, "dk": rdk, "dv": rdv}, TOL, "op3 rope")


@pytest.mark.parametrize("B,S,H,with_rope", [(2, 700, 3, False), (1, 680, 2, True),
                                             (1, 130, 1, True)])
def test_bf16_deterministic_backward_repeats_bit_identical(B, S, H, with_rope):
    """deterministic=1: three repeats give identical bits (the reference's
    gate, docs/TESTING.md:19 and bin/stability.rs:177-189), and the result
    is the op's gradient (oracle, 2e-2)."""
    from foundry_trainer_b200 import configs, ops
    g = torch.Generator().manual_seed(31 + S)
    shape = (B, S, H, 128)
    q, k, v = ((torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16).cuda() for _ in range(3))
    d_o = torch.randn(shape, generator=g).to(torch.bfloat16).cuda()
    pos = None
    rope = None
    if with_rope:
        pos = torch.zeros((S, 4))
        pos[:, 1] = torch.arange(S).float() // 24
        pos[:, 2] = torch.arange(S).float() % 24
        rope = ops.Rope(pos.cuda())
    o, lse = ops.attn_fwd(q, k, v, rope=rope)
    runs = [ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, deterministic=True) for _ in range(3)]
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for rep in runs[1:]:
        for name, a, b in zip(("dq", "dk", "dv"), runs[0], rep):
            assert torch.equal(a, b), name
    _, _, rdq, rdk, rdv = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "f32",
                                                rope_pos=pos.numpy() if pos is not None else None)
    assert_close({"dq": np32(runs[0][0]), "dk": np32(runs[0][1]), "dv": np32(runs[0][2])},
                 {"dq": rdq, "dk": rdk, "dv": rdv}, TOL, "deterministic")


@pytest.mark.parametrize("B,S,H", [(1, 1, 1), (1, 128, 2), (2, 130, 3), (1, 333, 2), (1, 1000, 2)])
def test_bf16_forward_in_tile_rotation_matches_rope_apply(B, S, H):
    """With RoPE inside, the forward rotates q and k in its tile loads and
    leaves them in its workspace for the backward. They are bit-identical to
    the standalone rotation (fa_rope_apply: the reference's apply_rope,
    lib.rs:122-129) at sizes with one, two, three (odd: a tile stored by two
    CTAs) and eight K tiles and ragged last tiles; O, LSE against the oracle."""
    from foundry_trainer_b200 import ops
    g = torch.Generator().manual_seed(41 + S)
    shape = (B, S, H, 128)
    q, k, v = ((torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16).cuda() for _ in range(3))
    pos = torch.zeros((S, 4))
    pos[:, 1] = torch.arange(S).float() // 20
    pos[:, 2] = torch.arange(S).float() % 20
    pos[:, 0] = (torch.arange(S) % 3).float()
    rope = ops.Rope(pos.cuda())
    saved = {}
    o, lse = ops.attn_fwd(q, k, v, rope=rope, saved=saved)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ws = saved["ws"]
    n = B * S * H * 128
    tb = (n * 2 + 255) // 256 * 256
    q_rot = ws[:n * 2].view(torch.bfloat16).view(shape)
    k_rot = ws[tb:tb + n * 2].view(torch.bfloat16).view(shape)
    assert torch.equal(q_rot, ops.rope_apply(q, rope))
    assert torch.equal(k_rot, ops.rope_apply(k, rope))
    # every K tile a CTA used, whether loaded rotated or rotated in its ring
    # slot, held the same bits: O equals the forward on pre-rotated inputs
    o_plain, lse_plain = ops.attn_fwd(ops.rope_apply(q, rope), ops.rope_apply(k, rope), v)
    torch.cuda.synchronize()
    assert torch.equal(o, o_plain) and torch.equal(lse, lse_plain)
    d_o = torch.zeros_like(q)
    ro, rlse, _, _, _ = orc.attn_fwd_bwd_bshd(np32(q), np32(k), np32(v), np32(d_o), "f32",
                                              rope_pos=pos.numpy())
    assert_close({"o": np32(o), "lse": np32(lse)}, {"o": ro, "lse": rlse}, TOL, "fused rope fwd")
