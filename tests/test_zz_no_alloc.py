"""fa_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some hosts cannot give the op a workspace at the call site — their memory
pool already owns the GPU, or cudaMalloc's device-wide synchronisation is not
acceptable on that path. fa_bwd_noalloc takes its scratch from a 64 MiB array
built into the library instead. This file checks, through the C ABI, that two
calls in a row give the same gradients as fa_bwd with a caller workspace
(within the bf16 tolerance the other tests use), and that sizes beyond the
array are refused with a clear error. It is collected last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes as C

import pytest
import torch

from oracle import attn_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 path tolerance (max |x - ref| / max |ref|)


def _inputs(B, S, H, seed):
    g = torch.Generator().manual_seed(seed)
    shape = (B, S, H, 128)
    q, k, v = ((torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16).cuda() for _ in range(3))
    d_o = torch.randn(shape, generator=g).to(torch.bfloat16).cuda()
    return q, k, v, d_o


def _noalloc(lib, q, k, v, o, d_o, lse, scale):
    from foundry_trainer_b200 import _lib
    from foundry_trainer_b200.ops import desc
    B, S, H, D = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ds = [desc(x) for x in (q, k, v, o, d_o, dq, dk, dv)]
    rc = lib.fa_bwd_noalloc(B, S, H, D, *[C.byref(x) for x in ds[:5]], lse.data_ptr(),
                            *[C.byref(x) for x in ds[5:]], scale,
                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "fa_bwd_noalloc")
    torch.cuda.synchronize()
    return dq, dk, dv


def test_noalloc_backward_matches_workspace_backward_twice():
    from foundry_trainer_b200 import _lib, ops
    lib = _lib.load()
    q, k, v, d_o = _inputs(1, 1000, 4, seed=77)
    scale = ops.default_scale(128)
    o, lse = ops.attn_fwd(q, k, v)
    ref = ops.attn_bwd(q, k, v, o, d_o, lse)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    _, _, odq, odk, odv = orc.attn_fwd_bwd_bshd(f(q), f(k), f(v), f(d_o), "f32")
    for call in range(2):
        got = _noalloc(lib, q, k, v, o, d_o, lse, scale)
        for name, a, b, r in zip(("dq", "dk", "dv"), got, ref, (odq, odk, odv)):
            err = orc.max_rel(f(a), f(b))
            assert err <= TOL, (call, name, "vs fa_bwd", err)
            err = orc.max_rel(f(a), r)
            assert err <= TOL, (call, name, "vs oracle", err)
    assert ops.device_status() == 0


def test_noalloc_refuses_sizes_beyond_its_array():
    from foundry_trainer_b200 import _lib
    from foundry_trainer_b200.ops import desc
    lib = _lib.load()
    # 1 x 8192 x 24 heads needs about 98 MiB of scratch: more than the 64 MiB array
    t = torch.empty((1, 16, 1, 128), device="cuda", dtype=torch.bfloat16)
    d = desc(t)
    lse = torch.empty(16, device="cuda")
    rc = lib.fa_bwd_noalloc(1, 8192, 24, 128, *[C.byref(d)] * 5, lse.data_ptr(),
                            *[C.byref(d)] * 3, 0.088, None)
    assert rc == _lib.FA_ERR_TOO_LARGE
    assert b"64 MiB" in lib.fa_last_error()


def test_noalloc_refuses_what_fa_bwd_refuses():
    import math

    from foundry_trainer_b200 import _lib
    from foundry_trainer_b200.ops import desc
    lib = _lib.load()
    t = torch.empty((1, 16, 1, 128), device="cuda", dtype=torch.bfloat16)
    d = desc(t)
    lse = torch.empty(16, device="cuda")
    call = lambda B, S, H, D, scale: lib.fa_bwd_noalloc(B, S, H, D, *[C.byref(d)] * 5,
                                                        lse.data_ptr(), *[C.byref(d)] * 3,
                                                        scale, None)
    for scale in (math.inf, math.nan, 0.0, -1.0):
        assert call(1, 16, 1, 128, scale) == _lib.FA_ERR_INVALID_ARG, scale
    assert call(1, 16, 1, 64, 0.088) == _lib.FA_ERR_UNSUPPORTED
    assert call(0, 16, 1, 128, 0.088) == _lib.FA_ERR_INVALID_ARG
    # the row padding is computed without int overflow: refused as too large
    assert call(1, 2**31 - 1, 1, 128, 0.088) == _lib.FA_ERR_TOO_LARGE
