"""The C ABI library loads and exports every entry point the header declares;
host-side validation answers without a GPU (no kernel is launched here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "foundry_attn.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(fa_\w+)\s*\(", text, re.M)))


def test_header_declarations_found():
    names = _declared()
    assert "fa_fwd" in names and "fa_bwd" in names and len(names) >= 12


def test_library_exports_every_declared_symbol():
    from foundry_trainer_b200 import _lib
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) <= set(_lib.SIGNATURES)


def test_status_strings_and_version():
    from foundry_trainer_b200 import _lib
    lib = _lib.load()
    assert lib.fa_abi_version() == 1
    for code in range(0, 9):
        assert lib.fa_status_string(code)
    assert _lib.status_string(0) == "ok"


def test_validation_rejects_bad_arguments_without_a_gpu():
    from foundry_trainer_b200 import _lib
    lib = _lib.load()
    t = _lib.fa_tensor_t(None, 0, 0, 0, 1)
    # null tensors
    rc = lib.fa_fwd(_lib.FA_DTYPE_BF16, 1, 16, 1, 128, C.byref(t), C.byref(t), C.byref(t),
                    C.byref(t), None, 0.1, None, None, 0, None)
    assert rc == _lib.FA_ERR_INVALID_ARG
    # unsupported head dim and dtype
    assert lib.fa_fwd(_lib.FA_DTYPE_BF16, 1, 16, 1, 64, None, None, None, None, None, 0.1, None,
                      None, 0, None) == _lib.FA_ERR_UNSUPPORTED
    assert lib.fa_fwd(7, 1, 16, 1, 128, None, None, None, None, None, 0.1, None, None, 0,
                      None) == _lib.FA_ERR_UNSUPPORTED
    # non-positive sizes
    assert lib.fa_bwd(_lib.FA_DTYPE_BF16, 0, 16, 1, 128, None, None, None, None, None, None, None,
                      None, None, 0.1, None, 0, None, 0, None) == _lib.FA_ERR_INVALID_ARG
    # a rotation whose axes do not cover the head dim
    r = _lib.fa_rope_t(1, 3, 32, 10000.0)
    assert lib.fa_rope_apply(_lib.FA_DTYPE_BF16, 1, 4, 1, 128, None, None, C.byref(r), 0,
                             None) == _lib.FA_ERR_UNSUPPORTED


def test_workspace_sizes():
    from foundry_trainer_b200 import _lib
    lib = _lib.load()
    B, S, H, D = 1, 4608, 24, 128
    assert lib.fa_fwd_workspace_bytes(_lib.FA_DTYPE_BF16, B, S, H, D, None) == 0
    r = _lib.fa_rope_t(1, 4, 32, 10000.0)
    assert lib.fa_fwd_workspace_bytes(_lib.FA_DTYPE_BF16, B, S, H, D, C.byref(r)) >= 2 * B * S * H * D * 2
    ws = lib.fa_bwd_workspace_bytes(_lib.FA_DTYPE_BF16, B, S, H, D, None, 0)
    assert ws >= B * S * H * D * 4 + 2 * B * H * S * 4


def test_loading_missing_library_fails_loudly(tmp_path, monkeypatch):
    from foundry_trainer_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(_lib.FaError):
        _lib.load()


def test_peer_exchange_entry_points_validate_without_a_gpu():
    from foundry_trainer_b200 import _lib
    lib = _lib.load()
    INV, ALIGN, TOO_LARGE = _lib.FA_ERR_INVALID_ARG, _lib.FA_ERR_ALIGNMENT, _lib.FA_ERR_TOO_LARGE
    assert lib.fa_peer_flags_bytes() >= 4 * (4 * 8 + 4)  # arrive[4][8] + epoch[4] words
    h = _lib.fa_peer_handle_t()
    p = C.c_void_p()
    assert lib.fa_peer_alloc(0, C.byref(p), C.byref(h)) == INV
    assert lib.fa_peer_open(None, C.byref(p)) == INV
    assert lib.fa_peer_close(None) == INV and lib.fa_peer_free(None) == INV
    # copies: nothing to do, null pointers, pitch below width, misalignment, rows
    assert lib.fa_copy_2d(None, 0, None, 0, 0, 1, None) == _lib.FA_OK
    assert lib.fa_copy_2d(None, 64, None, 64, 64, 1, None) == INV
    assert lib.fa_copy_2d(16, 32, 16, 64, 64, 1, None) == INV
    assert lib.fa_copy_2d_sm(16, 64, 24, 64, 64, 1, 4, None) == ALIGN
    assert lib.fa_copy_2d_sm(16, 64, 16, 64, 64, 70000, 4, None) == TOO_LARGE
    assert lib.fa_copy_2d_sm(16, 64, 16, 64, 64, 1, 0, None) == INV
    # barrier: world, rank and channel bounds, missing flag blocks
    flags = (C.c_void_p * 9)(*([4096] * 9))
    assert lib.fa_peer_barrier(0, 9, flags, 0, 1.0, None) == INV
    assert lib.fa_peer_barrier(2, 2, flags, 0, 1.0, None) == INV
    assert lib.fa_peer_barrier(0, 2, flags, 4, 1.0, None) == INV
    assert lib.fa_peer_barrier(0, 2, flags, 0, 0.0, None) == INV
    nul = (C.c_void_p * 2)(4096, None)
    assert lib.fa_peer_barrier(0, 2, nul, 0, 1.0, None) == INV
    assert lib.fa_peer_barrier(0, 1, flags, 0, 1.0, None) == _lib.FA_OK  # one rank: nothing
    # scatter: segments must cover the keys exactly once, at most 8
    t = _lib.fa_tensor_t(16, 0, 128, 128, 1)
    seg = (C.c_void_p * 9)(*([4096] * 9))
    args = lambda kv, s, n: (_lib.FA_DTYPE_BF16, 1, 256, kv, 1, 128, C.byref(t), C.byref(t),
                             C.byref(t), C.byref(t), 4096, 4096, 4096, s, n, seg, seg, 0.1, None)
    assert lib.fa_bwd_scatter(*args(512, 128, 2)) == INV    # 2 x 128 < 512 keys
    assert lib.fa_bwd_scatter(*args(512, 256, 3)) == INV    # a segment past the keys
    assert lib.fa_bwd_scatter(*args(2304, 256, 9)) == INV   # more than 8 segments
    assert lib.fa_bwd_scatter(_lib.FA_DTYPE_F32, 1, 256, 512, 1, 128, None, None, None, None,
                              None, None, None, 256, 2, seg, seg, 0.1,
                              None) == _lib.FA_ERR_UNSUPPORTED
    # reduce-cast and merge: head dim, parts, null and misaligned buffers
    y = _lib.fa_tensor_t(4096, 128 * 4, 128, 128, 1)
    assert lib.fa_reduce_cast_f32(_lib.FA_DTYPE_BF16, 1, 4, 1, 64, 4096, 4096, 2, 4096,
                                  C.byref(y), None, 1.0, None, None) == _lib.FA_ERR_UNSUPPORTED
    assert lib.fa_reduce_cast_f32(_lib.FA_DTYPE_BF16, 1, 4, 1, 128, 4096, 4096, 0, 4096,
                                  C.byref(y), None, 1.0, None, None) == INV
    assert lib.fa_reduce_cast_f32(_lib.FA_DTYPE_BF16, 1, 4, 1, 128, 4100, None, 2, 4096,
                                  C.byref(y), None, 1.0, None, None) == ALIGN
    assert lib.fa_merge_f32(_lib.FA_DTYPE_BF16, 1, 4, 1, 128, None, 4096, 4096, 4096,
                            C.byref(y), 4096, None) == INV
    assert lib.fa_merge_f32(_lib.FA_DTYPE_BF16, 1, 4, 1, 128, 4104, 4096, 4096, 4096,
                            C.byref(y), 4096, None) == ALIGN
