"""The callers of the attention op: the double- and single-stream DiT blocks
with LoRA, and the AdamW step on the LoRA factors.

Restates the reference's block code (crates/foundry-spike/src/lib.rs) over a
weight dictionary keyed like its fixtures and its `Weights` map
("weights/<name>.weight", ".bias", ".lora_a", ".lora_b"):

  linear            lib.rs:270-287  y = x W^T [+ b] + s * (x A^T) B^T
  swiglu            lib.rs:291-295  down(silu(gate(x)) * up(x))
  layer_norm_mod    lib.rs:60-71    LayerNorm in fp32, (1 + scale) * n + shift, cast
  double_block      lib.rs:301-392
  single_block      lib.rs:394-456
  single_block_fused bin/throughput.rs:577-629 (the klein single block)
  mse               lib.rs:458-463
  AdamW             lib.rs:472-505  fp32 moments, bias-corrected, weight decay 0
  checkpointed_backward lib.rs:519-638 (stage-wise recompute; attention
                    forward skipped with the kept O and LSE)

The attention of each block is a callable (`attention=`): by default the
B200 op with its fused q/k RMSNorm + RoPE prologue (`attn.JointAttention`
for the double block, `SingleAttention` here for the single block), which
take the per-stream projections before the norm and return the attention
output. Everything else (the linears, norms, modulation, MLPs) is torch on
the device: cuBLAS GEMMs and elementwise kernels.

Two block variants share this code:
  * the reference's (its fixtures and klein harness): one modulation linear
    for both streams of the double block (`<prefix>.mod`) or one per stream
    (`<prefix>.img.mod`, `<prefix>.txt.mod`, bin/throughput.rs:480-572),
    SwiGLU MLPs, optional biases;
  * the FLUX-style block of the LoRA benchmark configuration: modulation per
    stream, a 4x GELU (tanh) MLP `<prefix>.<stream>.mlp.fc1/.fc2`, LoRA on
    q/k/v/out of both streams (`make_c3_weights`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import attn, ops

Weights = Dict[str, torch.Tensor]

NORM_EPS = 1e-6  # lib.rs:26


def _get(w: Weights, key: str) -> torch.Tensor:
    t = w.get(key)
    if t is None:
        raise KeyError(f"weight missing: {key}")
    return t


# ------------------------------------------------------------------ ops

def linear(w: Weights, name: str, x: torch.Tensor, lora_scale: float) -> torch.Tensor:
    """x W^T (+ b) (+ lora_scale * (x A^T) B^T when the LoRA factors exist)."""
    y = F.linear(x, _get(w, f"weights/{name}.weight"))
    b = w.get(f"weights/{name}.bias")
    if b is not None:
        y = y + b
    a, bb = w.get(f"weights/{name}.lora_a"), w.get(f"weights/{name}.lora_b")
    if a is not None and bb is not None:
        y = y + F.linear(F.linear(x, a), bb) * lora_scale
    return y


def swiglu(w: Weights, name: str, x: torch.Tensor, lora_scale: float) -> torch.Tensor:
    gate = F.silu(linear(w, f"{name}.gate", x, lora_scale))
    up = linear(w, f"{name}.up", x, lora_scale)
    return linear(w, f"{name}.down", gate * up, lora_scale)


def gelu_mlp(w: Weights, name: str, x: torch.Tensor, lora_scale: float) -> torch.Tensor:
    """The FLUX MLP: fc2(gelu_tanh(fc1(x))), hidden 4x."""
    return linear(w, f"{name}.fc2", F.gelu(linear(w, f"{name}.fc1", x, lora_scale),
                                           approximate="tanh"), lora_scale)


def layer_norm_mod(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                   eps: float = NORM_EPS) -> torch.Tensor:
    xf = x.float()
    mean = xf.mean(dim=-1, keepdim=True)
    c = xf - mean
    var = (c * c).mean(dim=-1, keepdim=True)
    n = c / torch.sqrt(var + eps)
    return (n * (scale.float() + 1.0) + shift.float()).to(x.dtype)


def mse(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    d = a.float() - b.float()
    return (d * d).mean()


def _mlp(w: Weights, name: str, x: torch.Tensor, lora_scale: float) -> torch.Tensor:
    if f"weights/{name}.fc1.weight" in w:
        return gelu_mlp(w, name, x, lora_scale)
    return swiglu(w, name, x, lora_scale)


def modulation_sets(w: Weights, name: str, temb_silu: torch.Tensor, dim: int, sets: int,
                    lora_scale: float = 1.0) -> List[torch.Tensor]:
    """The 3*sets (dim,) chunks (shift, scale, gate per set) of
    linear(temb_silu) (bin/throughput.rs:297-324; lib.rs:310-317 with two
    sets). Constant across steps when temb is."""
    out = linear(w, name, temb_silu.reshape(1, dim), lora_scale).reshape(3 * sets * dim)
    return list(out.split(dim))


def _modulation(w: Weights, name: str, temb: torch.Tensor, dim: int,
                lora_scale: float) -> List[torch.Tensor]:
    """The six (dim,) chunks of linear(silu(temb)): shift1, scale1, gate1,
    shift2, scale2, gate2 (the reference feeds silu(temb), lib.rs:310-317)."""
    return modulation_sets(w, name, F.silu(temb), dim, 2, lora_scale)


# ------------------------------------------------------ attention callables

class SingleAttention:
    """Attention of the single-stream block (lib.rs:415-446) on the B200 op:
    q/k RMSNorm with their weights and RoPE at `positions` in one fused pass
    each (fa_qk_norm_rope_fwd with no text stream), the op, and the
    backward through both. (B, S, H, 128) bf16 in and out."""

    def __init__(self, positions: torch.Tensor, eps: float = NORM_EPS,
                 scale: Optional[float] = None):
        self.rope = ops.Rope(positions)
        self.eps = eps
        self.scale = scale

    def __call__(self, q, k, v, wq, wk):
        return _SingleAttention.apply(q, k, v, wq, wk, self.rope, self.eps, self.scale)


class _SingleAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, wq, wk, rope, eps, scale):
        q_r = ops.qk_norm_rope(None, q, None, wq, rope, eps=eps)
        k_r = ops.qk_norm_rope(None, k, None, wk, rope, eps=eps)
        v_c = v.contiguous()
        o, lse = ops.attn_fwd(q_r, k_r, v_c, scale=scale)
        ctx.save_for_backward(q, k, wq, wk, q_r, k_r, v_c, o, lse)
        ctx.rope, ctx.eps, ctx.scale = rope, eps, scale
        return o

    @staticmethod
    def backward(ctx, d_o):
        q, k, wq, wk, q_r, k_r, v_c, o, lse = ctx.saved_tensors
        dq_r, dk_r, dv = ops.attn_bwd(q_r, k_r, v_c, o, d_o.contiguous(), lse, scale=ctx.scale)
        _, dq, _, dwq = ops.qk_norm_rope_bwd(None, q, None, wq, ctx.rope, dq_r, eps=ctx.eps)
        _, dk, _, dwk = ops.qk_norm_rope_bwd(None, k, None, wk, ctx.rope, dk_r, eps=ctx.eps)
        return dq, dk, dv, dwq.to(wq.dtype), dwk.to(wk.dtype), None, None, None


class CheckpointedSingleAttention(SingleAttention):
    """SingleAttention for gradient-checkpointed blocks: keeps O and LSE in
    a graph-free forward and reuses them (no attention forward) in the
    recompute with gradients, like attn.CheckpointedJointAttention, and
    under the same check (attn.kept_matches on q, k, v and the two norm
    weights); any other call runs the full forward."""

    def __init__(self, positions: torch.Tensor, eps: float = NORM_EPS,
                 scale: Optional[float] = None):
        super().__init__(positions, eps, scale)
        self.kept = None

    def __call__(self, q, k, v, wq, wk):
        if not torch.is_grad_enabled():
            q_r = ops.qk_norm_rope(None, q, None, wq, self.rope, eps=self.eps)
            k_r = ops.qk_norm_rope(None, k, None, wk, self.rope, eps=self.eps)
            o, lse = ops.attn_fwd(q_r, k_r, v.contiguous(), scale=self.scale)
            self.kept = (o, lse, attn.kept_key((q, k, v), (wq, wk)))
            return o
        kept, self.kept = self.kept, None
        if kept is not None and attn.kept_matches(kept[2], (q, k, v), (wq, wk)):
            return _SingleAttentionReuse.apply(q, k, v, wq, wk, kept[:2], self.rope, self.eps,
                                               self.scale)
        return super().__call__(q, k, v, wq, wk)


class _SingleAttentionReuse(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, wq, wk, kept, rope, eps, scale):
        o, lse = kept  # a tuple: not an autograd input
        q_r = ops.qk_norm_rope(None, q, None, wq, rope, eps=eps)
        k_r = ops.qk_norm_rope(None, k, None, wk, rope, eps=eps)
        v_c = v.contiguous()
        ctx.save_for_backward(q, k, wq, wk, q_r, k_r, v_c, o, lse)
        ctx.rope, ctx.eps, ctx.scale = rope, eps, scale
        return o.view_as(o)

    @staticmethod
    def backward(ctx, d_o):
        return _SingleAttention.backward(ctx, d_o)[:5] + (None,) * 4


JointFn = Callable[..., Tuple[torch.Tensor, torch.Tensor]]
SingleFn = Callable[..., torch.Tensor]


# ---------------------------------------------------------------- blocks

@dataclass
class BlockShape:
    dim: int
    heads: int
    head_dim: int = 128


def double_block(w: Weights, img: torch.Tensor, txt: torch.Tensor, temb: torch.Tensor,
                 attention: JointFn, shape: BlockShape, *, prefix: str = "double",
                 lora_scale: float = 1.0,
                 acts: Optional[Dict[str, torch.Tensor]] = None,
                 mods: Optional[Tuple[List[torch.Tensor], List[torch.Tensor]]] = None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """One double-stream block (lib.rs:301-392). img (B, I, dim), txt (B, T,
    dim), temb (dim,). `attention(q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t,
    wq_i, wk_i)` gets the projections (B, len, H, head_dim) before the q/k
    RMSNorm and returns the (o_t, o_i) attention outputs. `mods` = the
    image and text streams' six modulation chunks when they are computed once
    for a whole stack (bin/throughput.rs:480-572); otherwise they come from
    this block's modulation linear(s)."""
    d, h, hd = shape.dim, shape.heads, shape.head_dim
    if mods is not None:
        mi, mt = mods
    elif f"weights/{prefix}.mod.weight" in w:
        mi = mt = _modulation(w, f"{prefix}.mod", temb, d, lora_scale)
    else:
        mi = _modulation(w, f"{prefix}.img.mod", temb, d, lora_scale)
        mt = _modulation(w, f"{prefix}.txt.mod", temb, d, lora_scale)
    B, I, T = img.shape[0], img.shape[1], txt.shape[1]

    ih = layer_norm_mod(img, mi[0], mi[1])
    th = layer_norm_mod(txt, mt[0], mt[1])
    if acts is not None:
        acts[f"{prefix}.img_norm1"], acts[f"{prefix}.txt_norm1"] = ih, th

    def proj(stream, x, n, which):
        return linear(w, f"{prefix}.{stream}.to_{which}", x, lora_scale).reshape(B, n, h, hd)

    q_i, k_i, v_i = (proj("img", ih, I, c) for c in ("q", "k", "v"))
    q_t, k_t, v_t = (proj("txt", th, T, c) for c in ("q", "k", "v"))
    a_t, a_i = attention(q_t, k_t, v_t, q_i, k_i, v_i,
                         _get(w, f"weights/{prefix}.txt_q_norm.weight"),
                         _get(w, f"weights/{prefix}.txt_k_norm.weight"),
                         _get(w, f"weights/{prefix}.img_q_norm.weight"),
                         _get(w, f"weights/{prefix}.img_k_norm.weight"))
    if acts is not None:
        acts[f"{prefix}.attn_img"] = a_i

    img = img + mi[2] * linear(w, f"{prefix}.img.to_out", a_i.reshape(B, I, d), lora_scale)
    txt = txt + mt[2] * linear(w, f"{prefix}.txt.to_out", a_t.reshape(B, T, d), lora_scale)
    if acts is not None:
        acts[f"{prefix}.img_post_attn"] = img

    ih2 = layer_norm_mod(img, mi[3], mi[4])
    th2 = layer_norm_mod(txt, mt[3], mt[4])
    img = img + mi[5] * _mlp(w, f"{prefix}.img.mlp", ih2, lora_scale)
    txt = txt + mt[5] * _mlp(w, f"{prefix}.txt.mlp", th2, lora_scale)
    if acts is not None:
        acts[f"{prefix}.img_out"], acts[f"{prefix}.txt_out"] = img, txt
    return img, txt


def single_block(w: Weights, x: torch.Tensor, temb: torch.Tensor, attention: SingleFn,
                 shape: BlockShape, *, prefix: str = "single", lora_scale: float = 1.0,
                 acts: Optional[Dict[str, torch.Tensor]] = None) -> torch.Tensor:
    """One single-stream block (lib.rs:394-456): fused QKV with LoRA, q/k
    RMSNorm + RoPE, attention, SwiGLU from the same normed input, gated
    residuals (x + g_at * attn + g_mlp * mlp; this block has no output
    projection and no second adaLN). x (B, S, dim); `attention(q, k, v, wq,
    wk)` gets the projections before the norm."""
    d, h, hd = shape.dim, shape.heads, shape.head_dim
    sh1, sc1, g_at, _, _, g_mlp = _modulation(w, f"{prefix}.mod", temb, d, lora_scale)
    B, S = x.shape[0], x.shape[1]
    nh = layer_norm_mod(x, sh1, sc1)
    if acts is not None:
        acts[f"{prefix}.norm1"] = nh
    qkv = linear(w, f"{prefix}.to_qkv", nh, lora_scale).reshape(B, S, 3, h, hd)
    q, k, v = qkv.unbind(2)
    o = attention(q, k, v, _get(w, f"weights/{prefix}.q_norm.weight"),
                  _get(w, f"weights/{prefix}.k_norm.weight"))
    a = o.reshape(B, S, d)
    if acts is not None:
        acts[f"{prefix}.attn"] = a
    m = _mlp(w, f"{prefix}.mlp", nh, lora_scale)
    if acts is not None:
        acts[f"{prefix}.mlp"] = m
    out = x + g_at * a + g_mlp * m
    if acts is not None:
        acts[f"{prefix}.out"] = out
    return out


def single_block_fused(w: Weights, x: torch.Tensor, mod3: List[torch.Tensor],
                       attention: SingleFn, shape: BlockShape, *, mlp_ratio: int = 3,
                       prefix: str = "single", lora_scale: float = 1.0) -> torch.Tensor:
    """The single-stream block in the klein layout (bin/throughput.rs:577-629):
    one fused in-projection `<prefix>.to_in` (dim -> (3 + 2*mlp_ratio)*dim:
    Q, K, V, then the SwiGLU gate and up of mlp_ratio*dim each), attention,
    silu(gate) * up, and one fused out-projection `<prefix>.to_out` over
    [attention | activation] (dim + mlp_ratio*dim -> dim); one gate on its
    output: x + g * out. mod3 = (shift, scale, gate)."""
    d, h, hd = shape.dim, shape.heads, shape.head_dim
    sh, sc, g = mod3
    B, S = x.shape[0], x.shape[1]
    nh = layer_norm_mod(x, sh, sc)
    fused = linear(w, f"{prefix}.to_in", nh, lora_scale).reshape(B, S, 3 + 2 * mlp_ratio, d)
    q, k, v = (fused[:, :, c].reshape(B, S, h, hd) for c in range(3))
    gate = fused[:, :, 3:3 + mlp_ratio].reshape(B, S, mlp_ratio * d)
    up = fused[:, :, 3 + mlp_ratio:].reshape(B, S, mlp_ratio * d)
    o = attention(q, k, v, _get(w, f"weights/{prefix}.q_norm.weight"),
                  _get(w, f"weights/{prefix}.k_norm.weight"))
    joined = torch.cat([o.reshape(B, S, d), F.silu(gate) * up], dim=-1)
    return x + g * linear(w, f"{prefix}.to_out", joined, lora_scale)


# ------------------------------------------ checkpointed forward/backward

Stage = Callable[[List[torch.Tensor]], List[torch.Tensor]]


def checkpointed_backward(stages: List[Stage], inputs: List[torch.Tensor],
                          seed: Callable[[List[torch.Tensor]], torch.Tensor],
                          params: List[torch.Tensor]):
    """Forward and backward keeping only each stage's inputs
    (lib.rs:519-638). Forward: every stage runs graph-free, so its
    intermediates are freed as it returns. Backward: stages in reverse; a
    stage's saved inputs become leaves, the stage runs again with gradients,
    and its upstream gradient enters through sum(out * upstream). Each
    parameter (a LoRA factor) must belong to exactly one stage. Attention
    callables that kept their O and LSE in the graph-free forward
    (attn.CheckpointedJointAttention, CheckpointedSingleAttention) skip the
    attention forward in the recompute.
    Returns (loss, input gradients, {id(param): gradient})."""
    if not stages:
        raise ValueError("checkpointed_backward: no stages")
    saved: List[List[torch.Tensor]] = []
    cur = [x.detach() for x in inputs]
    with torch.no_grad():
        for st in stages:
            saved.append(cur)
            cur = [o.detach() for o in st(cur)]
    outs = [o.requires_grad_(True) for o in cur]
    loss = seed(outs)
    upstream = list(torch.autograd.grad(loss, outs))
    param_grads = {}
    in_grads: List[torch.Tensor] = []
    for k in range(len(stages) - 1, -1, -1):
        leaves = [x.detach().requires_grad_(True) for x in saved[k]]
        with torch.enable_grad():
            o = stages[k](leaves)
            if len(o) != len(upstream):
                raise ValueError(f"stage {k} returned {len(o)} outputs, expected {len(upstream)}")
            seeded = sum((a * g).sum() for a, g in zip(o, upstream))
            g = torch.autograd.grad(seeded, leaves + params, allow_unused=True)
        for p, gp in zip(params, g[len(leaves):]):
            if gp is not None:
                param_grads[id(p)] = gp
        upstream = list(g[:len(leaves)])
        if k == 0:
            in_grads = upstream
    return loss.detach(), in_grads, param_grads


# ---------------------------------------------------------------- AdamW

@dataclass
class AdamW:
    """Bias-corrected AdamW, weight decay 0 (lib.rs:465-505): fp32 moments,
    step = lr * m_hat / (sqrt(v_hat) + eps), parameter updated in its own
    dtype."""
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8

    def init(self, params: List[torch.Tensor]) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        return [(torch.zeros_like(p, dtype=torch.float32),
                 torch.zeros_like(p, dtype=torch.float32)) for p in params]

    @torch.no_grad()
    def step(self, params: List[torch.Tensor], grads: List[torch.Tensor],
             state: List[Tuple[torch.Tensor, torch.Tensor]], t: int) -> None:
        bc1 = 1.0 - self.beta1 ** t
        bc2 = 1.0 - self.beta2 ** t
        for p, g, (m, v) in zip(params, grads, state):
            g = g.float()
            m.mul_(self.beta1).add_(g * (1.0 - self.beta1))
            v.mul_(self.beta2).add_(g * g * (1.0 - self.beta2))
            denom = torch.sqrt(v / bc2) + self.eps
            p.copy_((p.float() - (m / bc1) / denom * self.lr).to(p.dtype))


# ------------------------------------------- the benchmark configuration

def make_c3_weights(dim: int = 3072, heads: int = 24, rank: int = 16, seed: int = 0,
                    device=None, dtype=torch.bfloat16) -> Weights:
    """Random-init weights of the FLUX-style double block of the LoRA
    configuration: base weights ~N(0, 0.02), no biases, modulation per
    stream, q/k norm weights 1, a 4x GELU MLP per stream, LoRA rank `rank` on
    q/k/v/out of both streams with A ~N(0, 1/dim) and B = 0. Drawn from one
    CPU generator in key order, then moved."""
    g = torch.Generator().manual_seed(seed)
    w: Weights = {}

    def add(name, out_f, in_f, std=0.02):
        w[f"weights/{name}.weight"] = torch.randn(out_f, in_f, generator=g) * std

    for s in ("img", "txt"):
        add(f"double.{s}.mod", 6 * dim, dim)
        for c in ("q", "k", "v", "out"):
            add(f"double.{s}.to_{c}", dim, dim)
            w[f"weights/double.{s}.to_{c}.lora_a"] = (torch.randn(rank, dim, generator=g)
                                                      / math.sqrt(dim))
            w[f"weights/double.{s}.to_{c}.lora_b"] = torch.zeros(dim, rank)
        add(f"double.{s}.mlp.fc1", 4 * dim, dim)
        add(f"double.{s}.mlp.fc2", dim, 4 * dim)
        w[f"weights/double.{s}_q_norm.weight"] = torch.ones(128)
        w[f"weights/double.{s}_k_norm.weight"] = torch.ones(128)
    return {k: v.to(device=device, dtype=dtype) for k, v in w.items()}


def lora_keys(w: Weights) -> List[str]:
    return sorted(k for k in w if k.endswith(".lora_a") or k.endswith(".lora_b"))


def joint_positions(txt_len: int, grid: int) -> torch.Tensor:
    """(T + G*G, 4) axial positions of the joint sequence: text at 0, image
    token i at (0, i // G, i % G, 0)."""
    pos = torch.zeros((txt_len + grid * grid, 4), dtype=torch.float32)
    i = torch.arange(grid * grid)
    pos[txt_len:, 1] = (i // grid).float()
    pos[txt_len:, 2] = (i % grid).float()
    return pos


def allreduce_mean(grads, group=None):
    """Data-parallel replicas: the mean of each LoRA gradient over the ranks
    of `group`, with one all-reduce of one fp32 buffer."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = torch.cat([g.float().reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    flat /= world
    out, o = [], 0
    for g in grads:
        out.append(flat[o:o + g.numel()].view_as(g).to(g.dtype))
        o += g.numel()
    return out


class LoraTrainer:
    """One LoRA training step of a double block: forward, MSE loss against
    targets, backward to the LoRA factors only, AdamW. `attention` defaults
    to the B200 op (JointAttention at `positions`)."""

    def __init__(self, w: Weights, shape: BlockShape, positions: torch.Tensor, *,
                 lora_scale: float = 1.0, opt: Optional[AdamW] = None,
                 attention: Optional[JointFn] = None, grad_hook=None):
        self.w = dict(w)
        self.shape = shape
        self.lora_scale = lora_scale
        self.keys = lora_keys(w)
        self.params = [self.w[k] for k in self.keys]
        for p in self.params:
            p.requires_grad_(True)
        self.opt = opt if opt is not None else AdamW()
        self.state = self.opt.init(self.params)
        self.t = 0
        self.attention = attention if attention is not None else attn.JointAttention(
            positions.to(self.params[0].device))
        self.grad_hook = grad_hook  # e.g. an all-reduce of the LoRA grads across replicas

    def loss(self, img, txt, temb, target_img, target_txt):
        o_i, o_t = double_block(self.w, img, txt, temb, self.attention, self.shape,
                                lora_scale=self.lora_scale)
        return mse(o_i, target_img) + mse(o_t, target_txt)

    def step(self, img, txt, temb, target_img, target_txt) -> torch.Tensor:
        loss = self.loss(img, txt, temb, target_img, target_txt)
        grads = torch.autograd.grad(loss, self.params)
        if self.grad_hook is not None:
            grads = self.grad_hook(grads)
        self.t += 1
        self.opt.step(self.params, grads, self.state, self.t)
        return loss.detach()
