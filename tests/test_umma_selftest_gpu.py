"""Known-answer checks of the tcgen05 building blocks (descriptor layouts,
TMEM operand packing, MN-major operands, N=64 with a column offset).

Each case is one 128x128x128 bf16 product on one CTA, checked against an
fp32 torch matmul of the same bf16 values.
"""
import ctypes as C
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

SELFTEST = Path(__file__).resolve().parent / "lib" / "libfa_selftest.so"
_st = None


def _load():
    """tests/lib/libfa_selftest.so (built from tests/csrc/ by the package build)."""
    global _st
    if _st is None:
        if not SELFTEST.exists():
            raise RuntimeError(f"{SELFTEST} is missing; run `python -m foundry_trainer_b200.build`")
        st = C.CDLL(str(SELFTEST))
        st.fa_selftest_umma.restype = C.c_int
        st.fa_selftest_umma.argtypes = [C.c_int] + [C.c_void_p] * 5
        _st = st
    return _st


def _run(test_id, a, b):
    st = _load()
    d = torch.full((128, 128), float("nan"), device="cuda", dtype=torch.float32)
    status = torch.zeros(1, device="cuda", dtype=torch.int32)
    rc = st.fa_selftest_umma(test_id, a.data_ptr(), b.data_ptr(), d.data_ptr(), status.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return d


@pytest.mark.parametrize("test_id", [0, 1, 2, 3, 4])
def test_umma_known_answer(test_id):
    g = torch.Generator(device="cpu").manual_seed(100 + test_id)
    a = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    af, bf = a.float(), b.float()
    d = _run(test_id, a, b)
    if test_id == 0:
        ref = af @ bf.T
    elif test_id in (1, 2):
        ref = af @ bf
    elif test_id == 3:
        ref = af.T @ bf
    else:
        ref = af @ bf[:, 64:]
        d = d[:, 64:]
    err = (d - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, f"test {test_id}: max-rel {err}"
