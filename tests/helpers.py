"""Shared helpers for the GPU parity tests (checker side only)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import attn_oracle as orc


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def run_op(q, k, v, d_o, rope=None, scale=None):
    """Forward + backward through the C ABI; returns numpy float32 outputs."""
    from foundry_trainer_b200 import ops
    o, lse = ops.attn_fwd(q, k, v, rope=rope, scale=scale)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, scale=scale)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return tuple(np32(x) for x in (o, lse, dq, dk, dv))


def assert_close(ours: dict, ref: dict, tol: float, label: str = ""):
    errs = {n: orc.max_rel(ours[n], ref[n]) for n in ref}
    bad = {n: e for n, e in errs.items() if not (e <= tol)}
    assert not bad, f"{label} max-rel over {tol}: {bad} (all: {errs})"
    return errs
