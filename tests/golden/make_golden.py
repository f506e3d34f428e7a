"""Extracts the reference's attention golden vectors into small .npz fixtures.

Run once in a container that has the reference tree (it is not needed, and
not present, where the tests run):

    python tests/golden/make_golden.py /path/to/foundry-trainer

Sources (file:line in the reference):
  tools/fixtures/block_fp32.safetensors, block_bf16.safetensors — written by
  tools/fixtures/gen_block.py:374-385 (attention inputs `attn_in/*`, output,
  and `grad/attn/*`: dL/dq, dL/dk, dL/dv and the upstream gradient).

Outputs (float32 arrays; bf16 values are exact in float32):
  attn_fixture_fp32.npz, attn_fixture_bf16.npz
      {double,single}_{q,k,v,attn,dout,dq,dk,dv}: the isolated-op goldens the
      reference's own op test replays (src/bin/attn_backward.rs:203-233),
      S = 24 (8 text + 16 image), H = 2, D = 128.
  rope_fixture_fp32.npz, rope_fixture_bf16.npz
      {case}_pre, {case}_pos, {case}_post for the q/k rotations of both
      blocks: `post` is the reference's recorded post-RoPE tensor
      (double.q/double.k, attn_in/double.q[:8], single.q/single.k), `pre` is
      its input recomputed with the generator's own linear / LoRA / RMSNorm
      ops (gen_block.py:64-68, 129-131, 216-227, 273-276) from the recorded
      normalised activations and weights, and `pos` the generator's axial
      positions (gen_block.py:316-326, including the single block's
      image-then-text order).
  qk_norm_rope_fixture_fp32.npz, qk_norm_rope_fixture_bf16.npz
      x (the projection), w (the q-norm weight), pos, y = apply_rope(rms_norm(
      x, w)) and, for a seeded upstream gradient dy, dx and dw from torch
      autograd through the generator's ops (gen_block.py:65-69, 103-109).
  attn_rope_fixture_fp32.npz
      q, k, v (pre-rotation), dout, pos, and o, dq, dk, dv from the
      generator's own `apply_rope` + `attention` + torch autograd
      (gen_block.py:98-119) on seeded inputs: an end-to-end golden for the
      op with the rotation inside.
  block_fixture.npz
      the double + single block pair (weights, inputs, activations, loss,
      LoRA/input gradients, AdamW states) for the block replay (see
      block_fixture below).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    fx = Path(ref_root) / "tools" / "fixtures"
    sys.path.insert(0, str(fx))
    import gen_block as gb  # the reference's PyTorch semantics
    from safetensors.torch import load_file

    for tag, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        w = load_file(str(fx / f"block_{tag}.safetensors"))
        out = {}
        for blk in ("double", "single"):
            for n in ("q", "k", "v", "attn"):
                out[f"{blk}_{n}"] = w[f"attn_in/{blk}.{n}"].float().numpy()
            for n in ("q", "k", "v"):
                out[f"{blk}_d{n}"] = w[f"grad/attn/{blk}.{n}"].float().numpy()
            out[f"{blk}_dout"] = w[f"grad/attn/{blk}.out"].float().numpy()
        np.savez_compressed(HERE / f"attn_fixture_{tag}.npz", **out)

        # RoPE pins
        cfg = gb.CONFIG
        h, hd, eps = cfg["heads"], cfg["head_dim"], cfg["norm_eps"]
        lora_scale = cfg["lora_alpha"] / cfg["lora_rank"]

        def lin(name, x):
            y = torch.nn.functional.linear(x, w[f"weights/{name}.weight"], w[f"weights/{name}.bias"])
            if f"weights/{name}.lora_a" in w:
                y = y + lora_scale * torch.nn.functional.linear(
                    torch.nn.functional.linear(x, w[f"weights/{name}.lora_a"]),
                    w[f"weights/{name}.lora_b"])
            return y

        g = cfg["img_grid"]
        tl = cfg["txt_len"]
        rows = torch.arange(g * g) // g
        cols = torch.arange(g * g) % g
        z = torch.zeros(g * g)
        pos_img = torch.stack([rows.float(), cols.float(), z, z], dim=-1)
        zt = torch.zeros(tl)
        pos_txt = torch.stack([torch.arange(tl).float(), zt, zt, zt], dim=-1)
        pos_all = torch.cat([pos_img, pos_txt], dim=0)

        rope = {}
        ih = w["double.img_norm1"]
        th = w["double.txt_norm1"]
        cases = {
            "dimg_q": (lin("double.img.to_q", ih).view(-1, h, hd), "weights/double.img_q_norm.weight",
                       pos_img, w["double.q"]),
            "dimg_k": (lin("double.img.to_k", ih).view(-1, h, hd), "weights/double.img_k_norm.weight",
                       pos_img, w["double.k"]),
            "dtxt_q": (lin("double.txt.to_q", th).view(-1, h, hd), "weights/double.txt_q_norm.weight",
                       pos_txt, w["attn_in/double.q"][:tl]),
            "dtxt_k": (lin("double.txt.to_k", th).view(-1, h, hd), "weights/double.txt_k_norm.weight",
                       pos_txt, w["attn_in/double.k"][:tl]),
        }
        qkv = lin("single.to_qkv", w["single.norm1"]).view(-1, 3, h, hd)
        cases["single_q"] = (qkv[:, 0], "weights/single.q_norm.weight", pos_all, w["single.q"])
        cases["single_k"] = (qkv[:, 1], "weights/single.k_norm.weight", pos_all, w["single.k"])
        for name, (x, normw, pos, post) in cases.items():
            pre = gb.rms_norm(x, w[normw], eps)
            rope[f"{name}_pre"] = pre.float().numpy()
            rope[f"{name}_pos"] = pos.numpy().astype(np.float32)
            rope[f"{name}_post"] = post.float().numpy()
            # the RMSNorm input (the projection) and weight: with pos and
            # post, a golden of the fused QK-RMSNorm + RoPE prologue
            rope[f"{name}_h"] = x.float().numpy()
            rope[f"{name}_w"] = w[normw].float().numpy()
        np.savez_compressed(HERE / f"rope_fixture_{tag}.npz", **rope)

        # backward of the QK prologue: torch autograd through the generator's
        # rms_norm + apply_rope (gen_block.py:65-69, 103-109) for the double
        # block's image q case, with a seeded upstream gradient
        x, normw, pos, _ = cases["dimg_q"]
        cos, sin = gb.rope_tables(pos, cfg["rope_axes"], cfg["rope_theta"])
        xv = x.detach().clone().requires_grad_(True)
        wv = w[normw].detach().clone().requires_grad_(True)
        y = gb.apply_rope(gb.rms_norm(xv, wv, eps), cos, sin, cfg["rope_axes"])
        gen = torch.Generator().manual_seed(99)
        dy = torch.randn(y.shape, generator=gen).to(y.dtype)
        dx, dw = torch.autograd.grad(y, [xv, wv], dy)
        np.savez_compressed(HERE / f"qk_norm_rope_fixture_{tag}.npz",
                            x=x.float().numpy(), w=w[normw].float().numpy(),
                            pos=pos.numpy().astype(np.float32), y=y.detach().float().numpy(),
                            dy=dy.float().numpy(), dx=dx.float().numpy(), dw=dw.float().numpy())

    # end-to-end rotation-inside-the-op golden (fp32), seeded
    gen = torch.Generator().manual_seed(1234)
    txt, grid, H, D = 8, 4, 2, 128
    S = txt + grid * grid
    q = torch.randn(S, H, D, generator=gen)
    k = torch.randn(S, H, D, generator=gen)
    v = torch.randn(S, H, D, generator=gen)
    dout = torch.randn(S, H, D, generator=gen)
    i = torch.arange(grid * grid)
    pos = torch.zeros(S, 4)
    pos[txt:, 1] = (i // grid).float()
    pos[txt:, 2] = (i % grid).float()
    cos, sin = gb.rope_tables(pos, gb.CONFIG["rope_axes"], gb.CONFIG["rope_theta"])
    qv = q.clone().requires_grad_(True)
    kv = k.clone().requires_grad_(True)
    vv = v.clone().requires_grad_(True)
    qr = gb.apply_rope(qv, cos, sin, gb.CONFIG["rope_axes"])
    kr = gb.apply_rope(kv, cos, sin, gb.CONFIG["rope_axes"])
    o = gb.attention(qr, kr, vv)
    dq, dk, dv = torch.autograd.grad(o, [qv, kv, vv], dout)
    np.savez_compressed(HERE / "attn_rope_fixture_fp32.npz",
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), dout=dout.numpy(), pos=pos.numpy(),
                        o=o.detach().numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy())
    block_fixture(fx, gb)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


# activations the block replay compares (gen_block.py:199-247, 266-290, 361-362)
BLOCK_ACTS = ("double.img_norm1", "double.txt_norm1", "double.attn_img", "double.img_post_attn",
              "double.img_out", "double.txt_out", "single.norm1", "single.attn", "single.mlp",
              "single.out", "output/img", "output/txt", "loss")


def block_fixture(fx: Path, gb) -> None:
    """block_fixture.npz: the whole double + single block pair of the
    fixtures (gen_block.py:297-411) for a replay of the reference's block
    test (src/bin/block_backward.rs): the fp32 weights and inputs (the bf16
    run draws the same values and casts them, checked here), the recorded
    activations, loss, LoRA and input gradients and the AdamW states after 1
    and 10 steps of both runs (`<tag>:<key>`), and the axial positions.
    Keys use ':' where the fixture has '/'."""
    from safetensors.torch import load_file
    w32 = load_file(str(fx / "block_fp32.safetensors"))
    w16 = load_file(str(fx / "block_bf16.safetensors"))
    out = {}
    for k, t in w32.items():
        if k.startswith(("weights/", "inputs/")):
            assert torch.equal(w16[k], t.to(torch.bfloat16)), k
            out[k.replace("/", ":")] = t.numpy()
    for tag, src in (("fp32", w32), ("bf16", w16)):
        for k, t in src.items():
            if k in BLOCK_ACTS or k.startswith(("grad/double.", "grad/single.", "grad/inputs/",
                                                "opt1/", "opt10/")):
                out[f"{tag}:{k.replace('/', ':')}"] = t.float().numpy()
    cfg = gb.CONFIG
    g, tl = cfg["img_grid"], cfg["txt_len"]
    rows = torch.arange(g * g) // g
    cols = torch.arange(g * g) % g
    z = torch.zeros(g * g)
    zt = torch.zeros(tl)
    out["pos_img"] = torch.stack([rows.float(), cols.float(), z, z], dim=-1).numpy()
    out["pos_txt"] = torch.stack([torch.arange(tl).float(), zt, zt, zt], dim=-1).numpy()
    out["config"] = np.array([cfg["dim"], cfg["heads"], cfg["head_dim"], cfg["lora_rank"]],
                             dtype=np.int64)
    out["lora_scale"] = np.array(cfg["lora_alpha"] / cfg["lora_rank"], dtype=np.float64)
    out["adamw"] = np.array([cfg["lr"], *cfg["adamw_betas"], cfg["adamw_eps"]], dtype=np.float64)
    np.savez_compressed(HERE / "block_fixture.npz", **out)


if __name__ == "__main__":
    torch.use_deterministic_algorithms(True)
    torch.set_num_threads(1)
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
