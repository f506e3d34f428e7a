"""Tensor-level calls into the C ABI (PyTorch supplies device memory and streams).

Layouts follow the reference op: (S, H, D) per sequence as in
crates/foundry-spike/src/lib.rs:134, or batched (B, S, H, D). Any strides are
accepted as long as the head dimension is contiguous and the other strides
are 16-byte multiples (the TMA rule); nothing is copied to make inputs
contiguous.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import FA_DTYPE_BF16, FA_DTYPE_F32, check, fa_rope_t, fa_tensor_t

ROPE_AXES = (32, 32, 32, 32)  # lib.rs:20
ROPE_THETA = 10000.0          # lib.rs:21


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return FA_DTYPE_BF16
    if t.dtype == torch.float32:
        return FA_DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}: the op computes in bf16 or f32")


def as_bshd(t: torch.Tensor) -> torch.Tensor:
    """(S,H,D) -> (1,S,H,D) view; (B,S,H,D) unchanged."""
    if t.dim() == 3:
        return t.unsqueeze(0)
    if t.dim() == 4:
        return t
    raise ValueError(f"expected (S,H,D) or (B,S,H,D), got shape {tuple(t.shape)}")


def desc(t: torch.Tensor) -> fa_tensor_t:
    t4 = as_bshd(t)
    if not t4.is_cuda:
        raise ValueError("tensor must live on a CUDA device")
    sb, ss, sh, sd = t4.stride()
    return fa_tensor_t(t4.data_ptr(), sb, ss, sh, sd)


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


@dataclass
class Rope:
    """Axial RoPE descriptor: per-token positions (S, n_axes) and theta.

    Mirrors rope_tables_dtype (lib.rs:77-105); the tables are never
    materialised, the kernels evaluate cos/sin from the positions.
    """
    pos: torch.Tensor              # (S, n_axes) float32 on the device
    axis_dim: int = 32
    theta: float = ROPE_THETA

    def c_struct(self) -> fa_rope_t:
        p = self.pos
        if p.dtype != torch.float32 or not p.is_contiguous() or p.dim() != 2:
            raise ValueError("rope positions must be a contiguous (S, n_axes) float32 tensor")
        return fa_rope_t(p.data_ptr(), p.shape[1], self.axis_dim, self.theta)


def _ref(x):
    return C.byref(x) if x is not None else None


def default_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)  # lib.rs:138


def attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
             rope: Optional[Rope] = None, out: Optional[torch.Tensor] = None,
             lse: Optional[torch.Tensor] = None, stream=None, saved: Optional[dict] = None):
    """O and fp32 LSE (B, H, S) of softmax(Q K^T * scale) V.

    With `rope` and a `saved` dict, the forward's workspace (rotated q, k and
    their (cos, sin) table) is kept in it for attn_bwd(..., saved=...), which
    then skips the second rotation."""
    q4, k4, v4 = as_bshd(q), as_bshd(k), as_bshd(v)
    B, S, H, D = q4.shape
    if k4.shape != q4.shape or v4.shape != q4.shape:
        raise ValueError("q, k, v must share one shape")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share one dtype")
    dt = _dtype_code(q)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((B, H, S), device=q.device, dtype=torch.float32)
    scale = default_scale(D) if scale is None else float(scale)
    lib = _lib.load()
    rc_rope = rope.c_struct() if rope is not None else None
    ws_bytes = lib.fa_fwd_workspace_bytes(dt, B, S, H, D, _ref(rc_rope))
    ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8) if ws_bytes else None
    if saved is not None:
        saved.clear()
        if ws is not None:
            saved.update(ws=ws, shape=(B, S, H, D), dtype=q.dtype)
    dq_, dk_, dv_, do_ = desc(q4), desc(k4), desc(v4), desc(as_bshd(out))
    check(lib.fa_fwd(dt, B, S, H, D, C.byref(dq_), C.byref(dk_), C.byref(dv_), C.byref(do_),
                     lse.data_ptr(), scale, _ref(rc_rope), ws.data_ptr() if ws is not None else None,
                     ws_bytes, _stream_ptr(stream)), "fa_fwd")
    return out, lse


def attn_bwd(q, k, v, o, d_o, lse, *, scale: Optional[float] = None, rope: Optional[Rope] = None,
             deterministic: bool = False, dq=None, dk=None, dv=None, stream=None,
             saved: Optional[dict] = None):
    """dQ, dK, dV of the op (w.r.t. pre-rotation q/k when rope is given).

    `saved`: the dict a matching attn_fwd(..., saved=...) filled; the bf16
    path then reuses the forward's rotated q, k (fa_bwd_saved)."""
    q4 = as_bshd(q)
    B, S, H, D = q4.shape
    dt = _dtype_code(q)
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    scale = default_scale(D) if scale is None else float(scale)
    lib = _lib.load()
    rc_rope = rope.c_struct() if rope is not None else None
    if (saved and rope is not None and dt == FA_DTYPE_BF16 and not deterministic
            and saved.get("shape") == (B, S, H, D) and saved.get("dtype") == q.dtype):
        fws = saved["ws"]
        ws_bytes = lib.fa_bwd_saved_workspace_bytes(dt, B, S, H, D)
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        ds = [desc(x) for x in (v, o, d_o, dq, dk, dv)]
        check(lib.fa_bwd_saved(dt, B, S, H, D, fws.data_ptr(), fws.numel(),
                               *[C.byref(x) for x in ds[:3]], lse.data_ptr(),
                               *[C.byref(x) for x in ds[3:]], scale, C.byref(rc_rope),
                               ws.data_ptr(), ws_bytes, _stream_ptr(stream)), "fa_bwd_saved")
        return dq, dk, dv
    ws_bytes = lib.fa_bwd_workspace_bytes(dt, B, S, H, D, _ref(rc_rope), int(deterministic))
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    ds = [desc(x) for x in (q, k, v, o, d_o, dq, dk, dv)]
    check(lib.fa_bwd(dt, B, S, H, D, *[C.byref(x) for x in ds[:5]], lse.data_ptr(),
                     *[C.byref(x) for x in ds[5:]], scale, _ref(rc_rope), int(deterministic),
                     ws.data_ptr(), ws_bytes, _stream_ptr(stream)), "fa_bwd")
    return dq, dk, dv


def rope_apply(x: torch.Tensor, rope: Rope, *, inverse: bool = False, out=None, stream=None):
    """The reference's apply_rope (lib.rs:122-129) on the device."""
    x4 = as_bshd(x)
    B, S, H, D = x4.shape
    out = torch.empty_like(x) if out is None else out
    r = rope.c_struct()
    dx, dy = desc(x), desc(out)
    check(_lib.load().fa_rope_apply(_dtype_code(x), B, S, H, D, C.byref(dx), C.byref(dy),
                                    C.byref(r), int(inverse), _stream_ptr(stream)),
          "fa_rope_apply")
    return out


NORM_EPS = 1e-6  # lib.rs:26


def qk_norm_rope(x_txt: Optional[torch.Tensor], x_img: Optional[torch.Tensor],
                 w_txt: Optional[torch.Tensor], w_img: Optional[torch.Tensor],
                 rope: Optional[Rope], *, eps: float = NORM_EPS,
                 out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """The joint block's fused q/k prologue (fa_qk_norm_rope_fwd): per stream
    rms_norm with its weight (lib.rs:45-58), apply_rope with the joint
    positions (lib.rs:122-129), written text-then-image into one
    (B, T+I, H, 128) tensor (the cat of lib.rs:363-365). Either stream may
    be None; bf16."""
    xs = [x for x in (x_txt, x_img) if x is not None]
    if not xs:
        raise ValueError("at least one stream is required")
    t4 = as_bshd(x_txt) if x_txt is not None else None
    i4 = as_bshd(x_img) if x_img is not None else None
    B, _, H, D = as_bshd(xs[0]).shape
    T = t4.shape[1] if t4 is not None else 0
    I = i4.shape[1] if i4 is not None else 0
    if out is None:
        out = torch.empty((B, T + I, H, D), device=xs[0].device, dtype=xs[0].dtype)
    r = rope.c_struct() if rope is not None else None
    dt_ = desc(t4) if t4 is not None else None
    di_ = desc(i4) if i4 is not None else None
    do_ = desc(out)
    check(_lib.load().fa_qk_norm_rope_fwd(
        _dtype_code(xs[0]), B, T, I, H, D, _ref(dt_), _ref(di_),
        w_txt.data_ptr() if w_txt is not None else None,
        w_img.data_ptr() if w_img is not None else None, float(eps), _ref(r), C.byref(do_),
        _stream_ptr(stream)), "fa_qk_norm_rope_fwd")
    return out


def qk_norm_rope_bwd(x_txt, x_img, w_txt, w_img, rope: Optional[Rope], dy: torch.Tensor, *,
                     eps: float = NORM_EPS, dw_txt: Optional[torch.Tensor] = None,
                     dw_img: Optional[torch.Tensor] = None, stream=None):
    """Gradients of qk_norm_rope: (dx_txt, dx_img, dw_txt, dw_img). The weight
    gradients are fp32 and ADDED to dw_* when given (zeros otherwise)."""
    t4 = as_bshd(x_txt) if x_txt is not None else None
    i4 = as_bshd(x_img) if x_img is not None else None
    d4 = as_bshd(dy)
    B, S, H, D = d4.shape
    T = t4.shape[1] if t4 is not None else 0
    I = i4.shape[1] if i4 is not None else 0
    dev = dy.device
    dx_t = torch.empty_like(x_txt) if x_txt is not None else None
    dx_i = torch.empty_like(x_img) if x_img is not None else None
    if x_txt is not None and dw_txt is None:
        dw_txt = torch.zeros(D, device=dev, dtype=torch.float32)
    if x_img is not None and dw_img is None:
        dw_img = torch.zeros(D, device=dev, dtype=torch.float32)
    r = rope.c_struct() if rope is not None else None
    ds = [desc(x) if x is not None else None for x in (t4, i4, d4, dx_t, dx_i)]
    check(_lib.load().fa_qk_norm_rope_bwd(
        _dtype_code(dy), B, T, I, H, D, _ref(ds[0]), _ref(ds[1]),
        w_txt.data_ptr() if w_txt is not None else None,
        w_img.data_ptr() if w_img is not None else None, float(eps), _ref(r), C.byref(ds[2]),
        _ref(ds[3]), _ref(ds[4]), dw_txt.data_ptr() if dw_txt is not None else None,
        dw_img.data_ptr() if dw_img is not None else None, _stream_ptr(stream)),
        "fa_qk_norm_rope_bwd")
    return dx_t, dx_i, dw_txt, dw_img


def device_status() -> int:
    """Reads and clears the device status word (0 when no bounded wait expired)."""
    return int(_lib.load().fa_device_status())
