"""Host-side mirror of the reference's attention custom op.

The reference implements `AttnBwd` as a Candle `CustomOp3`
(crates/foundry-spike/src/lib.rs:151-264) and calls it as
`q.apply_op3(&k, &v, AttnBwd)` (lib.rs:366, 444). This module keeps that
surface — `name()`, `cpu_fwd`, `cuda_fwd`, `bwd(q, k, v, res, grad_res)` and
`apply_op3` — over the B200 C ABI, so a caller (and a test written like the
reference's `bin/attn_backward.rs`) swaps the op without other changes.

Differences from the reference, by design:
  * `cpu_fwd` raises: the B200 op has no CPU fallback (the reference's CPU
    arithmetic lives only in the test oracle, `oracle/`).
  * `cuda_fwd` saves the fp32 log-sum-exp; `bwd` consumes it instead of
    recomputing softmax (lib.rs:232-238).
  * optional `scale` (the reference hard-codes 1/sqrt(head_dim), lib.rs:138)
    and `rope` (rotation inside the op; the reference rotates before it).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops
from ._lib import FaError


def _tensor_key(q: torch.Tensor, k: torch.Tensor):
    """Identity of the (q, k) a forward rotated: storage, layout and version."""
    return (q.data_ptr(), tuple(q.stride()), q._version, k.data_ptr(), tuple(k.stride()),
            k._version)


class AttnBwd:
    """The joint-attention op, CustomOp3-shaped (lib.rs:151-264)."""

    def __init__(self, scale: Optional[float] = None, rope: Optional[ops.Rope] = None,
                 deterministic: bool = False):
        self.scale = scale
        self.rope = rope
        self.deterministic = deterministic
        self._saved_lse: Optional[torch.Tensor] = None
        # with rope: the forward's rotated q, k and (cos, sin) table, reused by bwd
        self._saved_fwd: dict = {}

    def name(self) -> str:
        return "foundry-attn-bwd"  # lib.rs:154-156

    def cpu_fwd(self, q, k, v):
        raise FaError(2, "AttnBwd::cpu_fwd",
                      "the B200 attention op has no CPU path; move q/k/v to a CUDA device")

    def cuda_fwd(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Forward on device storage (lib.rs:189-214); keeps the LSE for bwd."""
        out, lse = ops.attn_fwd(q, k, v, scale=self.scale, rope=self.rope,
                                saved=self._saved_fwd)
        self._saved_fwd["key"] = _tensor_key(q, k)
        self._saved_lse = lse
        return out

    def bwd(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, res: torch.Tensor,
            grad_res: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dq, dk, dv) given the forward output `res` and its gradient (lib.rs:216-263)."""
        lse = self._saved_lse
        if lse is None:
            # Called without a preceding cuda_fwd on this instance: rebuild the
            # statistics with one forward pass.
            _, lse = ops.attn_fwd(q, k, v, scale=self.scale, rope=self.rope)
        # the forward's rotated q, k are reused only for the very tensors it saw
        saved = self._saved_fwd if self._saved_fwd.get("key") == _tensor_key(q, k) else None
        return ops.attn_bwd(q, k, v, res, grad_res.contiguous(), lse, scale=self.scale,
                            rope=self.rope, deterministic=self.deterministic, saved=saved)

    def fwd(self, q, k, v):
        if q.is_cuda:
            return self.cuda_fwd(q, k, v)
        return self.cpu_fwd(q, k, v)


class _Op3(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, op: AttnBwd):
        out = op.fwd(q, k, v)
        ctx.op = op
        ctx.lse = op._saved_lse
        ctx.saved_fwd = dict(op._saved_fwd)
        ctx.save_for_backward(q, k, v, out)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out = ctx.saved_tensors
        op: AttnBwd = ctx.op
        op._saved_lse = ctx.lse
        op._saved_fwd = ctx.saved_fwd
        dq, dk, dv = op.bwd(q, k, v, out, grad_out)
        return dq, dk, dv, None


def apply_op3(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, op: AttnBwd) -> torch.Tensor:
    """`q.apply_op3(&k, &v, op)`: forward now, op.bwd under autograd."""
    return _Op3.apply(q, k, v, op)


class _JointAttention(torch.autograd.Function):
    """The double block's attention with its fused prologue (see JointAttention)."""

    @staticmethod
    def forward(ctx, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i, rope, eps, scale):
        T = q_t.shape[1]
        q_j = ops.qk_norm_rope(q_t, q_i, wq_t, wq_i, rope, eps=eps)
        k_j = ops.qk_norm_rope(k_t, k_i, wk_t, wk_i, rope, eps=eps)
        v_j = ops.qk_norm_rope(v_t, v_i, None, None, None)  # concatenation only
        o_j, lse = ops.attn_fwd(q_j, k_j, v_j, scale=scale)
        ctx.save_for_backward(q_t, k_t, q_i, k_i, wq_t, wk_t, wq_i, wk_i, q_j, k_j, v_j, o_j, lse)
        ctx.rope, ctx.eps, ctx.scale, ctx.T = rope, eps, scale, T
        # the narrow of lib.rs:367-368: views of the joint output
        return o_j[:, :T], o_j[:, T:]

    @staticmethod
    def backward(ctx, do_t, do_i):
        return _joint_backward(ctx, do_t, do_i) + (None, None, None)


def _joint_backward(ctx, do_t, do_i):
    """Gradients of the ten tensor inputs of the joint attention from the
    saved prologue inputs, the joint q/k/v, O and LSE."""
    (q_t, k_t, q_i, k_i, wq_t, wk_t, wq_i, wk_i, q_j, k_j, v_j, o_j,
     lse) = ctx.saved_tensors
    T = ctx.T
    do_j = ops.qk_norm_rope(do_t.contiguous(), do_i.contiguous(), None, None, None)
    dq_j, dk_j, dv_j = ops.attn_bwd(q_j, k_j, v_j, o_j, do_j, lse, scale=ctx.scale)
    dq_t, dq_i, dwq_t, dwq_i = ops.qk_norm_rope_bwd(q_t, q_i, wq_t, wq_i, ctx.rope, dq_j,
                                                    eps=ctx.eps)
    dk_t, dk_i, dwk_t, dwk_i = ops.qk_norm_rope_bwd(k_t, k_i, wk_t, wk_i, ctx.rope, dk_j,
                                                    eps=ctx.eps)
    cast = lambda g, w: g.to(w.dtype) if g is not None else None
    return (dq_t, dk_t, dv_j[:, :T], dq_i, dk_i, dv_j[:, T:], cast(dwq_t, wq_t),
            cast(dwk_t, wk_t), cast(dwq_i, wq_i), cast(dwk_i, wk_i))


class _JointAttentionReuse(torch.autograd.Function):
    """The joint attention with O and LSE given (kept from an earlier,
    graph-free forward on the same inputs): the prologue runs again for the
    backward's joint q/k/v, the attention forward does not."""

    @staticmethod
    def forward(ctx, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i, kept, rope, eps,
                scale):
        # `kept` = (O, LSE) as a tuple: not an autograd input, so the outputs
        # are views of a tensor this node owns, as in _JointAttention
        o_j, lse = kept
        T = q_t.shape[1]
        q_j = ops.qk_norm_rope(q_t, q_i, wq_t, wq_i, rope, eps=eps)
        k_j = ops.qk_norm_rope(k_t, k_i, wk_t, wk_i, rope, eps=eps)
        v_j = ops.qk_norm_rope(v_t, v_i, None, None, None)
        ctx.save_for_backward(q_t, k_t, q_i, k_i, wq_t, wk_t, wq_i, wk_i, q_j, k_j, v_j, o_j, lse)
        ctx.rope, ctx.eps, ctx.scale, ctx.T = rope, eps, scale, T
        return o_j[:, :T], o_j[:, T:]

    @staticmethod
    def backward(ctx, do_t, do_i):
        return _joint_backward(ctx, do_t, do_i) + (None, None, None, None)


class JointAttention:
    """Attention of the double-stream block from the two streams'
    projections, as the reference composes it (lib.rs:326-368):
    per stream q/k RMSNorm with that stream's weights, axial RoPE with the
    joint positions, cat([txt, img]), the AttnBwd op, and the txt/img narrow.
    Here the norm, the rotation and the concatenation are one fused pass
    (fa_qk_norm_rope_fwd) per tensor writing the joint tensor the attention
    kernels read; the outputs are views of the joint O. Differentiable in the
    six projections and the four norm weights. bf16, (B, len, H, 128)."""

    def __init__(self, positions: torch.Tensor, eps: float = ops.NORM_EPS,
                 scale: Optional[float] = None):
        self.rope = ops.Rope(positions)
        self.eps = eps
        self.scale = scale

    def __call__(self, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i):
        return _JointAttention.apply(q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i,
                                     self.rope, self.eps, self.scale)


_PROBE_ROWS = 64


def kept_key(inputs, weights):
    """Identity of one call's inputs, stored with the O and LSE a graph-free
    forward keeps and compared by `kept_matches` before they are reused.

    The recompute of a checkpointed stage makes fresh projection tensors
    (new storage, possibly at an address an unrelated tensor held before),
    so storage addresses cannot tell the recompute of the same forward from
    another call. The key holds instead: each input's shape, dtype and
    device; each weight's storage and version (the weights are the same
    tensors, unchanged, between a forward and its recompute); and an exact
    copy of about 64 evenly spaced sequence rows of each input (all heads and
    head-dim entries of those rows)."""
    def probe(t):
        t = t.detach()
        step = max(1, t.shape[1] // _PROBE_ROWS)
        return t[:, ::step].clone()

    return (tuple((tuple(t.shape), t.dtype, t.device) for t in inputs),
            tuple((w.data_ptr(), w._version, tuple(w.shape)) for w in weights),
            tuple(probe(t) for t in inputs))


def kept_matches(key, inputs, weights) -> bool:
    """True when `inputs` / `weights` are, by kept_key's test, those the key
    was taken from (one device synchronisation for the row comparison)."""
    if key is None:
        return False
    meta, wid, probes = key
    if meta != tuple((tuple(t.shape), t.dtype, t.device) for t in inputs):
        return False
    if wid != tuple((w.data_ptr(), w._version, tuple(w.shape)) for w in weights):
        return False
    now = kept_key(inputs, ())[2]
    return all(torch.equal(a, b) for a, b in zip(probes, now))


class CheckpointedJointAttention(JointAttention):
    """JointAttention for gradient-checkpointed blocks: in a graph-free
    forward (torch.no_grad) it keeps the joint O and LSE; the next call with
    gradients enabled — the block's recompute during the checkpointed
    backward, on the same inputs — reuses them and skips the attention
    forward (the LSE makes the recompute unnecessary; the backward needs only
    O, LSE and the joint q/k/v). The kept values are reused only when the
    call's inputs pass `kept_matches` against the forward's (shapes, the
    weights' identity and version, exact sampled rows of the six
    projections); any other call runs the full forward. Each block should
    have its own instance (a shared one is correct, but keeps only the last
    forward's values)."""

    def __init__(self, positions: torch.Tensor, eps: float = ops.NORM_EPS,
                 scale: Optional[float] = None):
        super().__init__(positions, eps, scale)
        self.kept = None

    def __call__(self, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i):
        if not torch.is_grad_enabled():
            q_j = ops.qk_norm_rope(q_t, q_i, wq_t, wq_i, self.rope, eps=self.eps)
            k_j = ops.qk_norm_rope(k_t, k_i, wk_t, wk_i, self.rope, eps=self.eps)
            v_j = ops.qk_norm_rope(v_t, v_i, None, None, None)
            o_j, lse = ops.attn_fwd(q_j, k_j, v_j, scale=self.scale)
            self.kept = (o_j, lse, kept_key((q_t, k_t, v_t, q_i, k_i, v_i),
                                            (wq_t, wk_t, wq_i, wk_i)))
            T = q_t.shape[1]
            return o_j[:, :T], o_j[:, T:]
        kept, self.kept = self.kept, None
        if kept is not None and kept_matches(kept[2], (q_t, k_t, v_t, q_i, k_i, v_i),
                                             (wq_t, wk_t, wq_i, wk_i)):
            return _JointAttentionReuse.apply(q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i,
                                              wk_i, kept[:2], self.rope, self.eps, self.scale)
        return super().__call__(q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i)
