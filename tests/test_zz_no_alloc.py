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
    for call in range(2):
        got = _noalloc(lib, q, k, v, o, d_o, lse, scale)
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            err = orc.max_rel(a.float().cpu().numpy(), b.float().cpu().numpy())
            assert err <= TOL, (call, name, err)
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
