"""ctypes binding of the C ABI in include/foundry_attn.h.

The library is the product path: there is no CPU or PyTorch fallback. If
`lib/libfoundry_attn.so` is missing, loading raises instead of degrading.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "lib" / "libfoundry_attn.so"

FA_OK = 0
FA_ERR_INVALID_ARG = 1
FA_ERR_UNSUPPORTED = 2
FA_ERR_ALIGNMENT = 3
FA_ERR_LAUNCH = 4
FA_ERR_DEVICE_TIMEOUT = 5
FA_ERR_WORKSPACE = 6
FA_ERR_NO_DEVICE = 7
FA_ERR_TOO_LARGE = 8

FA_DTYPE_F32 = 0
FA_DTYPE_BF16 = 1


class FaError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {message} (status {status})")
        self.status = status


class fa_tensor_t(C.Structure):
    _fields_ = [("data", C.c_void_p), ("stride_b", C.c_int64), ("stride_s", C.c_int64),
                ("stride_h", C.c_int64), ("stride_d", C.c_int64)]


class fa_rope_t(C.Structure):
    _fields_ = [("pos", C.c_void_p), ("n_axes", C.c_int), ("axis_dim", C.c_int),
                ("theta", C.c_float)]


class fa_peer_handle_t(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


_T = C.POINTER(fa_tensor_t)
_R = C.POINTER(fa_rope_t)
_F = C.c_void_p  # float* (device)

# name -> (restype, argtypes)
SIGNATURES = {
    "fa_fwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T, _T, _F,
                         C.c_float, _R, C.c_void_p, C.c_size_t, C.c_void_p]),
    "fa_fwd_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _R]),
    "fa_bwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T, _T, _T, _F,
                         _T, _T, _T, C.c_float, _R, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "fa_bwd_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _R,
                                            C.c_int]),
    "fa_bwd_saved": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                               C.c_size_t, _T, _T, _T, _F, _T, _T, _T, C.c_float, _R,
                               C.c_void_p, C.c_size_t, C.c_void_p]),
    "fa_bwd_saved_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "fa_qk_norm_rope_fwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T,
                                      C.c_void_p, C.c_void_p, C.c_float, _R, _T, C.c_void_p]),
    "fa_qk_norm_rope_bwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T,
                                      C.c_void_p, C.c_void_p, C.c_float, _R, _T, _T, _T, _F, _F,
                                      C.c_void_p]),
    "fa_rope_apply": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _R, C.c_int,
                                C.c_void_p]),
    "fa_fwd_partial": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T,
                                 _T, _F, C.c_float, C.c_void_p]),
    "fa_fwd_fold": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T,
                              _F, _F, C.c_int, C.c_int, _T, _F, C.c_float, C.c_void_p]),
    "fa_lse_merge": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _F, _F, _T, _F,
                               C.c_int, C.c_void_p]),
    "fa_bwd_prepare": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _F, _F, _F,
                                 C.c_void_p]),
    "fa_bwd_partial": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T,
                                 _T, _F, _F, _F, _F, _F, C.c_int, C.c_float, C.c_void_p]),
    "fa_add_f32": (C.c_int, [C.c_int64, _F, _F, C.c_void_p]),
    "fa_cast_f32": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _F, C.c_int, _T,
                              C.c_float, _R, C.c_void_p]),
    "fa_bwd_noalloc": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T, _T, _T, _F, _T, _T,
                                 _T, C.c_float, C.c_void_p]),
    "fa_peer_flags_bytes": (C.c_size_t, []),
    "fa_peer_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), C.POINTER(fa_peer_handle_t)]),
    "fa_peer_open": (C.c_int, [C.POINTER(fa_peer_handle_t), C.POINTER(C.c_void_p)]),
    "fa_peer_close": (C.c_int, [C.c_void_p]),
    "fa_peer_free": (C.c_int, [C.c_void_p]),
    "fa_copy_2d": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t,
                             C.c_size_t, C.c_void_p]),
    "fa_copy_2d_sm": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t,
                                C.c_size_t, C.c_int, C.c_void_p]),
    "fa_peer_barrier": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_void_p), C.c_int, C.c_double,
                                  C.c_void_p]),
    "fa_bwd_scatter": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _T, _T, _T,
                                 _T, _F, _F, _F, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                 C.POINTER(C.c_void_p), C.c_float, C.c_void_p]),
    "fa_reduce_cast_f32": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _F, _F, C.c_int,
                                     C.c_int64, _T, _T, C.c_float, _R, C.c_void_p]),
    "fa_merge_f32": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _F, _F, _F, _F, _T, _F,
                               C.c_void_p]),
    "fa_timing_enable": (C.c_int, [C.c_int]),
    "fa_timing_read": (C.c_int, [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int)]),
    "fa_status_string": (C.c_char_p, [C.c_int]),
    "fa_last_error": (C.c_char_p, []),
    "fa_device_status": (C.c_int, []),
    "fa_abi_version": (C.c_int, []),
    "fa_build_info": (C.c_char_p, []),
}

_lib = None


def load() -> C.CDLL:
    """Loads libfoundry_attn.so (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FaError(-1, "load", f"{LIB_PATH} is missing; run `python -m foundry_trainer_b200.build`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().fa_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != FA_OK:
        msg = status_string(status)
        if status == FA_ERR_LAUNCH:
            msg += f" [{load().fa_last_error().decode()}]"
        raise FaError(status, where, msg)


def loaded_path() -> str:
    return os.fspath(LIB_PATH)
