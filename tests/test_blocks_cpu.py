"""The block callers of the attention op (foundry_trainer_b200.blocks)
replayed against the reference's recorded double + single block pair
(tests/golden/block_fixture.npz, from tools/fixtures/block_{fp32,bf16}
.safetensors), on CPU with the torch stand-in for the B200 attention
(tests/block_support.py): the block code around the op — LoRA linears,
adaLN modulation, SwiGLU, gated residuals, the joint sequence, MSE loss,
backward to the LoRA factors, AdamW — against the reference's activations,
gradients and optimiser states (its block test, src/bin/block_backward.rs,
and optimiser test, src/bin/opt_step.rs).

Forward activations, loss and gradients: fp32 rel-L2 <= 1e-5 (same
arithmetic up to association; measured <= 1e-6), bf16 rel-L2 <= 1e-3
(measured: bit-identical). AdamW states: fp32 updates rel-L2 <= 1e-3; bf16
the reference's own comparison, cos >= 0.999 and rel-L2 <= 2e-2
(crates/foundry-spike/src/lib.rs:640-667) — the generator's optimiser keeps
bf16 moments, the reference's Rust step (and this one) fp32 moments.
"""
import pytest
import torch

from foundry_trainer_b200 import blocks
from tests import block_support as bs

ACTS = ("double.img_norm1", "double.txt_norm1", "double.attn_img", "double.img_post_attn",
        "double.img_out", "double.txt_out", "single.norm1", "single.attn", "single.mlp",
        "single.out", "output/img", "output/txt")


def _check(tag, name, ours, ref, tight=True):
    ours = ours.detach().float().reshape(ref.shape)
    if tight:
        tol = 1e-5 if tag == "fp32" else 1e-3
        assert bs.rel_l2(ours, ref) <= tol, (name, bs.rel_l2(ours, ref))
    else:
        assert bs.cosine(ours, ref) >= 0.999 and bs.rel_l2(ours, ref) <= 2e-2, (
            name, bs.cosine(ours, ref), bs.rel_l2(ours, ref))


@pytest.fixture(scope="module")
def fx():
    return bs.Fixture()


def _run(fx, tag):
    dtype = torch.float32 if tag == "fp32" else torch.bfloat16
    return bs.FixtureRun(fx, dtype, "cpu", lambda p: bs.TorchJointAttention(p, dtype),
                         lambda p: bs.TorchSingleAttention(p, dtype))


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_block_pair_forward_and_lora_grads_match_reference(fx, tag):
    run = _run(fx, tag)
    acts, grads = run.grads()
    for name in ACTS:
        _check(tag, name, acts[name][0], fx.recorded(tag, name))
    # the recorded bf16 loss is the bf16-rounded mse; this one stays fp32 (lib.rs:458-463)
    _check(tag, "loss", acts["loss"].reshape(1), fx.recorded(tag, "loss").reshape(1),
           tight=tag == "fp32")
    lora = [k for k in fx.z.files if k.startswith(f"{tag}:grad:")]
    assert len(lora) == 8  # 3 LoRA linears x (A, B) + the two input gradients
    for key in lora:
        name = key[len(tag) + 1:].replace(":", "/")
        _check(tag, name, grads[name], fx.recorded(tag, name))


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_adamw_on_lora_matches_reference_steps(fx, tag):
    run = _run(fx, tag)
    hist = run.train(10)
    for step in (1, 10):
        for k in run.lora:
            name = k[len("weights/"):]
            ref = fx.recorded(tag, f"opt{step}/{name}")
            ours = hist[step - 1][k]
            if tag == "fp32":
                # the update is lr * m_hat / (sqrt(v_hat) + eps): compare the change
                init = fx.get(k)
                assert bs.rel_l2(ours.float() - init, ref - init) <= 1e-3, (step, name)
            else:
                _check(tag, f"opt{step}/{name}", ours, ref, tight=False)


def test_double_block_variants_and_lora_init():
    # the FLUX-style weights of the LoRA configuration at a small width: per
    # stream modulation, GELU MLP, LoRA B = 0 so the first step's A-gradients
    # vanish and the outputs do not depend on A
    torch.manual_seed(0)
    w = blocks.make_c3_weights(dim=256, heads=2, rank=4, seed=3, dtype=torch.float32)
    assert all(float(w[k].abs().max()) == 0.0 for k in w if k.endswith(".lora_b"))
    shape = blocks.BlockShape(dim=256, heads=2)
    pos = blocks.joint_positions(8, 4)
    attn_ = bs.TorchJointAttention(pos, torch.float32)
    g = torch.Generator().manual_seed(1)
    img, txt = torch.randn(1, 16, 256, generator=g), torch.randn(1, 8, 256, generator=g)
    temb, ti, tt = torch.randn(256, generator=g), torch.randn(1, 16, 256, generator=g), \
        torch.randn(1, 8, 256, generator=g)
    tr = blocks.LoraTrainer(w, shape, pos, attention=attn_)
    loss0 = tr.loss(img, txt, temb, ti, tt)
    keys = tr.keys
    grads = torch.autograd.grad(loss0, tr.params)
    for k, gk in zip(keys, grads):
        if k.endswith(".lora_a"):
            assert float(gk.abs().max()) == 0.0, k
        else:
            assert float(gk.abs().max()) > 0.0, k
    losses = [float(tr.step(img, txt, temb, ti, tt)) for _ in range(5)]
    assert losses[-1] < losses[0]


def test_product_attention_fails_loudly_on_cpu():
    from foundry_trainer_b200 import attn
    w = blocks.make_c3_weights(dim=256, heads=2, rank=4, seed=3, dtype=torch.bfloat16)
    pos = blocks.joint_positions(8, 4)
    img, txt = torch.zeros(1, 16, 256, dtype=torch.bfloat16), torch.zeros(1, 8, 256,
                                                                          dtype=torch.bfloat16)
    with pytest.raises(Exception):
        blocks.double_block(w, img, txt, torch.zeros(256, dtype=torch.bfloat16),
                            attn.JointAttention(pos), blocks.BlockShape(256, 2))


def test_single_block_fused_layout():
    # the klein single block against a direct composition of its parts
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
    mod3 = blocks.modulation_sets(w, "mod_single", torch.nn.functional.silu(temb), d, 1)
    att = bs.TorchSingleAttention(blocks.joint_positions(8, 4), torch.float32)
    out = blocks.single_block_fused(w, x, mod3, att, shape, mlp_ratio=mr, prefix="single.0")

    sh, sc, gt = mod3
    nh = blocks.layer_norm_mod(x, sh, sc)
    W_in = w["weights/single.0.to_in.weight"] + (w["weights/single.0.to_in.lora_b"]
                                                 @ w["weights/single.0.to_in.lora_a"])
    fused = nh @ W_in.T
    q, k, v = (fused[..., i * d:(i + 1) * d].reshape(1, S, h, 128) for i in range(3))
    gate, up = fused[..., 3 * d:(3 + mr) * d], fused[..., (3 + mr) * d:]
    o = att(q, k, v, w["weights/single.0.q_norm.weight"], w["weights/single.0.k_norm.weight"])
    ref = x + gt * (torch.cat([o.reshape(1, S, d), torch.nn.functional.silu(gate) * up], -1)
                    @ w["weights/single.0.to_out.weight"].T)
    assert bs.rel_l2(out, ref) <= 1e-5


def test_checkpointed_backward_matches_autograd_on_the_block_pair(fx):
    # the reference's stage-wise checkpointing (lib.rs:519-638) over the
    # fixture's double and single block: same loss, LoRA and input gradients
    # as one autograd pass
    dtype = torch.float32
    run = _run(fx, "fp32")
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

    loss, in_grads, pg = blocks.checkpointed_backward([double, single], [run.img, run.txt],
                                                       seed, params)
    acts, ref = run.grads()
    assert bs.rel_l2(loss.reshape(1), acts["loss"].reshape(1)) <= 1e-6
    assert bs.rel_l2(in_grads[0][0], ref["grad/inputs/img"]) <= 1e-6
    assert bs.rel_l2(in_grads[1][0], ref["grad/inputs/txt"]) <= 1e-6
    for k, p in zip(run.lora, params):
        assert bs.rel_l2(pg[id(p)], ref["grad/" + k[len("weights/"):]]) <= 1e-6, k


def test_data_parallel_lora_replicas_on_gloo_match_averaged_gradients():
    import multiprocessing as mp
    import socket
    world, steps = 2, 3
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=bs.dp_gloo_rank, args=(r, world, port, steps, results))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, grads, params = results.get(timeout=240)
            got[r] = ([torch.from_numpy(g) for g in grads],
                      {k: torch.from_numpy(v) for k, v in params.items()})
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    # the all-reduced first-step gradient is the mean of the replicas' own
    # (recomputed here in one process); AdamW's first update is about
    # lr * sign(g), so the factors themselves are compared between replicas,
    # which apply the same averaged gradients and must stay identical
    tr, batches = bs.dp_problem(world)
    per = [torch.autograd.grad(tr.loss(*b), tr.params) for b in batches]
    mean = [sum(gs) / world for gs in zip(*per)]
    for i, k in enumerate(tr.keys):
        for r in range(world):
            assert bs.rel_l2(got[r][0][i], mean[i]) <= 1e-5, (r, k)
    assert all(torch.equal(got[0][1][k], got[1][1][k]) for k in tr.keys)
    assert any(not torch.equal(got[0][1][k], p.detach()) for k, p in zip(tr.keys, tr.params))


def test_kept_attention_values_are_reused_only_for_the_same_inputs():
    # the guard of the checkpointed attention callables (attn.kept_key /
    # kept_matches): equal inputs in fresh tensors match (the checkpointed
    # recompute); another shape, another weight version, or a changed
    # sampled row do not (a stale kept O/LSE is never reused)
    from foundry_trainer_b200 import attn
    g = torch.Generator().manual_seed(4)
    xs = [torch.randn(1, 300, 2, 128, generator=g) for _ in range(3)]
    ws = [torch.rand(128, generator=g) for _ in range(2)]
    key = attn.kept_key(xs, ws)
    assert attn.kept_matches(key, [x.clone() for x in xs], ws)
    assert not attn.kept_matches(None, xs, ws)
    assert not attn.kept_matches(key, [xs[0][:, :299]] + xs[1:], ws)
    assert not attn.kept_matches(key, xs, [ws[0].clone(), ws[1]])  # another weight tensor
    ws[1].mul_(1.0)  # same values, new version: the weights may have been updated
    assert not attn.kept_matches(key, xs, ws)
    key = attn.kept_key(xs, ws)
    changed = [x.clone() for x in xs]
    changed[2][0, 0, 1, 5] += 1.0  # row 0 is sampled
    assert not attn.kept_matches(key, changed, ws)
