"""The C++ CustomOp3 mirror (include/foundry_attn_op.hpp) checked against the
CPU oracle through its compiled driver (tests/cpp/test_attn_op.cpp)."""
import subprocess

import numpy as np
import pytest

from oracle import attn_oracle as orc
from foundry_trainer_b200 import build as fbuild

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,with_rope", [("bf16", True), ("f32", False)])
def test_cpp_mirror_fwd_bwd(tmp_path, dtype, with_rope):
    from foundry_trainer_b200 import configs
    drv = fbuild.LIB / "test_attn_op"
    assert drv.exists(), "C++ driver not built"
    txt, grid, H = 32, 8, 2
    pos = configs.positions(txt, grid).numpy()
    S = pos.shape[0]
    rng = np.random.default_rng(21)
    arrs = {n: (rng.standard_normal((S, H, 128)) * (0.5 if n != "do" else 1.0)).astype(np.float32)
            for n in ("q", "k", "v", "do")}
    if dtype == "bf16":
        arrs = {n: orc.bf16_round(a) for n, a in arrs.items()}
    for n, a in arrs.items():
        a.tofile(tmp_path / f"{n}.bin")
    pos.astype(np.float32).tofile(tmp_path / "pos.bin")
    cmd = [str(drv), str(tmp_path), dtype, str(S), str(H)] + (["rope"] if with_rope else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    ours = {n: np.fromfile(tmp_path / f"{n}.bin", dtype=np.float32).reshape(S, H, 128)
            for n in ("o", "dq", "dk", "dv")}
    ref = orc.attn_fwd_bwd_bshd(arrs["q"][None], arrs["k"][None], arrs["v"][None],
                                arrs["do"][None], "f32", rope_pos=pos if with_rope else None)
    tol = 2e-2 if dtype == "bf16" else 1e-4
    for name, r_ in zip(("o", "dq", "dk", "dv"), (ref[0][0], ref[2][0], ref[3][0], ref[4][0])):
        assert orc.max_rel(ours[name], r_) <= tol, name
