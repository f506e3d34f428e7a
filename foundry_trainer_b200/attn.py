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
