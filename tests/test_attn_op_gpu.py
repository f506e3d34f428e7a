"""The CustomOp3-shaped mirror, exercised the way the reference tests its op
(src/bin/attn_backward.rs:190-239): wrap the fixture's q/k/v as leaves, run
the op, compare the forward output, seed the backward with the recorded
upstream gradient through `sum(attn * seed)`, compare dq/dk/dv with the
reference's acceptance metric (cos >= 0.999 and rel-L2 <= 2e-2)."""
import numpy as np
import pytest
import torch

from oracle import attn_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tag,dtype", [("bf16", torch.bfloat16), ("fp32", torch.float32)])
def test_attn_backward_like_reference(golden_dir, tag, dtype):
    from foundry_trainer_b200.attn import AttnBwd, apply_op3
    g = dict(np.load(golden_dir / f"attn_fixture_{tag}.npz"))
    for blk in ("double", "single"):
        q, k, v = (torch.from_numpy(g[f"{blk}_{n}"]).to(dtype).cuda().requires_grad_(True)
                   for n in ("q", "k", "v"))
        op = AttnBwd()
        assert op.name() == "foundry-attn-bwd"
        attn = apply_op3(q, k, v, op)
        cos, rel = orc.compare(attn.detach().float().cpu().numpy(), g[f"{blk}_attn"])
        assert cos >= 0.999 and rel <= 2e-2, ("fwd", blk)
        seed = torch.from_numpy(g[f"{blk}_dout"]).to(dtype).cuda()
        (attn * seed).float().sum().backward()
        for n, var in (("q", q), ("k", k), ("v", v)):
            cos, rel = orc.compare(var.grad.float().cpu().numpy(), g[f"{blk}_d{n}"])
            assert cos >= 0.999 and rel <= 2e-2, (blk, n, cos, rel)


def test_cpu_fwd_has_no_fallback():
    from foundry_trainer_b200._lib import FaError
    from foundry_trainer_b200.attn import AttnBwd
    x = torch.zeros(4, 1, 128)
    with pytest.raises(FaError):
        AttnBwd().fwd(x, x, x)
