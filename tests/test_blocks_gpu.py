"""The block callers of the op with the B200 attention inside, on the GPU.

* The reference's recorded double + single block pair (its block tests,
  crates/foundry-spike/src/bin/block_forward.rs / block_backward.rs;
  tests/golden/block_fixture.npz) replayed in bf16 with the fused q/k
  prologue and the sm_100a attention kernels (attn.JointAttention,
  blocks.SingleAttention): activations, loss, LoRA and input gradients
  against the recorded bf16 values under the reference's acceptance metric,
  cos >= 0.999 and rel-L2 <= 2e-2 (lib.rs:640-667).
* The checkpointed backward (lib.rs:519-638) with the checkpointed attention
  callables, which keep O and LSE in the graph-free forward and skip the
  attention forward in the recompute: the same loss and gradients as one
  autograd pass, with the forward kernel launched once per block.
* The kept-value guard on the device: a graph-free call on other inputs is
  never reused.
* The klein single block's fused projections (bin/throughput.rs:577-629)
  against the same block on CPU in fp32 with the torch stand-in attention.
"""
import pytest
import torch

from foundry_trainer_b200 import attn, blocks
from tests import block_support as bs
from tests.test_blocks_cpu import ACTS

pytestmark = pytest.mark.gpu


def _ok(a, b):
    a = a.detach().float().cpu().reshape(b.shape)
    return bs.cosine(a, b) >= 0.999 and bs.rel_l2(a, b) <= 2e-2, (bs.cosine(a, b),
                                                                 bs.rel_l2(a, b))


@pytest.fixture(scope="module")
def fx():
    return bs.Fixture()


def _b200_run(fx, checkpointed=False):
    joint = attn.CheckpointedJointAttention if checkpointed else attn.JointAttention
    single = blocks.CheckpointedSingleAttention if checkpointed else blocks.SingleAttention
    return bs.FixtureRun(fx, torch.bfloat16, "cuda", lambda p: joint(p.cuda()),
                         lambda p: single(p.cuda()))


def test_block_pair_replay_with_b200_attention(fx):
    run = _b200_run(fx)
    acts, grads = run.grads()
    torch.cuda.synchronize()
    for name in ACTS:
        ok, m = _ok(acts[name][0], fx.recorded("bf16", name))
        assert ok, (name, m)
    ok, m = _ok(acts["loss"].reshape(1), fx.recorded("bf16", "loss").reshape(1))
    assert ok, ("loss", m)
    lora = [k for k in fx.z.files if k.startswith("bf16:grad:")]
    assert len(lora) == 8
    for key in lora:
        name = key[len("bf16:"):].replace(":", "/")
        ok, m = _ok(grads[name], fx.recorded("bf16", name))
        assert ok, (name, m)


def _count_forward_launches(monkeypatch):
    from foundry_trainer_b200 import ops
    calls = []
    real = ops.attn_fwd

    def counting(*a, **k):
        calls.append(1)
        return real(*a, **k)

    monkeypatch.setattr(ops, "attn_fwd", counting)
    return calls


def test_checkpointed_backward_reuses_o_lse_and_matches_autograd(fx, monkeypatch):
    ref_run = _b200_run(fx)
    acts, ref = ref_run.grads()
    run = _b200_run(fx, checkpointed=True)
    params = [run.w[k] for k in run.lora]
    for p in params:
        p.requires_grad_(True)

    def double(xs):
        img2, txt2 = blocks.double_block(run.w, xs[0], xs[1], run.temb, run.joint, fx.shape,
                                         lora_scale=fx.lora_scale)
        return [torch.cat([txt2, img2], dim=1)]

    def single(xs):
        return [blocks.single_block(run.w, xs[0], run.temb, run.single, fx.shape,
                                    lora_scale=fx.lora_scale)]

    def seed(outs):
        o = outs[0]
        return blocks.mse(o[:, run.T:], run.target_img) + blocks.mse(o[:, :run.T], run.target_txt)

    calls = _count_forward_launches(monkeypatch)
    loss, in_grads, pg = blocks.checkpointed_backward([double, single], [run.img, run.txt],
                                                       seed, params)
    torch.cuda.synchronize()
    # one attention forward per block (the graph-free pass); the recompute reused O, LSE
    assert len(calls) == 2, len(calls)
    ok, m = _ok(loss.reshape(1), acts["loss"].detach().float().cpu().reshape(1))
    assert ok, ("loss", m)
    for i, n in enumerate(("img", "txt")):
        ok, m = _ok(in_grads[i][0], ref[f"grad/inputs/{n}"].float().cpu())
        assert ok, (n, m)
    for k, p in zip(run.lora, params):
        ok, m = _ok(pg[id(p)], ref["grad/" + k[len("weights/"):]].float().cpu())
        assert ok, (k, m)


def test_checkpointed_attention_never_reuses_values_of_other_inputs(monkeypatch):
    torch.manual_seed(3)
    T, G, H = 8, 4, 2
    pos = blocks.joint_positions(T, G).cuda()
    mk = lambda n: (torch.randn(1, n, H, 128, device="cuda") * 0.5).to(torch.bfloat16)
    w = [torch.rand(128, device="cuda").to(torch.bfloat16) + 0.5 for _ in range(4)]
    xs = [mk(T), mk(T), mk(T), mk(G * G), mk(G * G), mk(G * G)]
    ys = [mk(T), mk(T), mk(T), mk(G * G), mk(G * G), mk(G * G)]
    ck = attn.CheckpointedJointAttention(pos)
    with torch.no_grad():
        ck(*xs, *w)  # keeps O, LSE of xs
    calls = _count_forward_launches(monkeypatch)
    got = ck(*[y.requires_grad_(True) for y in ys], *w)  # other inputs: full forward
    assert len(calls) == 1
    ref = attn.JointAttention(pos)(*ys, *w)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    # the values of a graph-free call on the same inputs are reused
    with torch.no_grad():
        ck(*ys, *w)
    calls.clear()
    again = ck(*ys, *w)
    assert len(calls) == 0
    for a, b in zip(again, ref):
        assert torch.equal(a, b)


def test_single_block_fused_on_b200_matches_cpu_fp32():
    torch.manual_seed(5)
    d, h, mr, S = 256, 2, 3, 24
    shape = blocks.BlockShape(dim=d, heads=h)
    g = torch.Generator().manual_seed(7)
    w = {"weights/single.0.to_in.weight": torch.randn((3 + 2 * mr) * d, d, generator=g) * 0.02,
         "weights/single.0.to_in.lora_a": torch.randn(4, d, generator=g) * 0.02,
         "weights/single.0.to_in.lora_b": torch.randn((3 + 2 * mr) * d, 4, generator=g) * 0.02,
         "weights/single.0.to_out.weight": torch.randn(d, d + mr * d, generator=g) * 0.02,
         "weights/single.0.q_norm.weight": torch.rand(128, generator=g) + 0.5,
         "weights/single.0.k_norm.weight": torch.rand(128, generator=g) + 0.5,
         "weights/mod_single.weight": torch.randn(3 * d, d, generator=g) * 0.02}
    x = torch.randn(1, S, d, generator=g)
    temb = torch.randn(d, generator=g)
    pos = blocks.joint_positions(8, 4)

    def run(dev, dtype, att):
        ww = {k: t.to(device=dev, dtype=dtype) for k, t in w.items()}
        xx, tt = x.to(device=dev, dtype=dtype), temb.to(device=dev, dtype=dtype)
        mod3 = blocks.modulation_sets(ww, "mod_single", torch.nn.functional.silu(tt), d, 1)
        return blocks.single_block_fused(ww, xx, mod3, att, shape, mlp_ratio=mr,
                                         prefix="single.0")

    ref = run("cpu", torch.float32, bs.TorchSingleAttention(pos, torch.float32))
    out = run("cuda", torch.bfloat16, blocks.SingleAttention(pos.cuda()))
    torch.cuda.synchronize()
    ok, m = _ok(out, ref)
    assert ok, m
