"""ctypes binding of libglaucis_b200.so (declared in include/glaucis_b200.h).

The product path loads the in-tree shared library and nothing else: if it is
missing or fails to load, every op raises instead of computing elsewhere.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libglaucis_b200.so"
_lock = threading.Lock()
_lib = None

GL_OK = 0
GL_EINVAL = -1
GL_ELAUNCH = -2
GL_EDEVICE = -3
GL_OUT_BF16 = 0
GL_OUT_F32 = 1
GL_GLA_BF16_INTRA = 1
DEV_CODES = {0: "ok", 1: "device wait timed out", 2: "invalid group_sizes (negative or sum > M)"}

# (name, restype, argtypes) for every symbol the header declares.
_P, _I64, _I, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "gl_quant_act_1x128": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "gl_quant_w_128x128": (_I, [_P, _I64, _I64, _I64, _P, _P, _P, _P]),
    "gl_gmm_fp8_fwd": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _P]),
    "gl_chunk_gla_fwd": (_I, [_P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64, _I64,
                              _P, _P, _P, _P]),
    "gl_chunk_gla_fwd_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I64, _I64]),
    "gl_chunk_gla_fwd_ws": (_I, [_P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64, _I64,
                                 _P, _P, _P, ctypes.c_size_t, _P, _P]),
    "gl_chunk_gla_fwd_states": (_I, [_P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64,
                                     _I64, _P, _P, _P, _P, ctypes.c_size_t, _P, _P]),
    "gl_chunk_gla_fwd_ex": (_I, [_P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64, _I64,
                                 _P, _P, _P, _P, ctypes.c_size_t, _I, _P, _P]),
    "gl_chunk_gla_fwd_scatter": (_I, [_P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64,
                                      _I64, _P, _I, _P, _P, ctypes.c_size_t, _I, _P, _P]),
    "gl_chunk_gla_fwd_intermediates": (_I, [_P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64, _P,
                                            _P, _P, _P]),
    "gl_chunk_gla_bwd_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I64, _I64]),
    "gl_chunk_gla_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _I64, _I64,
                              _I64, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P]),
    "gl_gmm_fp8_fwd_scatter": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I, _I64, _I,
                                    _P, _P]),
    "gl_ipc_alloc": (_I, [ctypes.c_size_t, _P, _P]),
    "gl_ipc_open": (_I, [_P, _P]),
    "gl_ipc_close": (_I, [_P]),
    "gl_ipc_free": (_I, [_P]),
    "gl_gmm_fp8_act_fwd_noalloc": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _P]),
    "gl_quant_col_128x1": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "gl_gmm_fp8_dlhs": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _P]),
    "gl_tgmm_fp8": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I, _P, _P]),
    "gl_device_status": (_I, [_P, _P, ctypes.POINTER(ctypes.c_int)]),
    "gl_last_error": (ctypes.c_char_p, []),
    "gl_version": (ctypes.c_char_p, []),
}


class GlaucisError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def lib_path() -> Path:
    return _LIB_PATH


def load(build_if_missing: bool = False):
    """Returns the loaded library, raising if the shared object is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists() and build_if_missing:
            from . import build as _build
            _build.build()
        if not _LIB_PATH.exists():
            raise GlaucisError(
                f"{_LIB_PATH} is missing: run `python -m glaucis_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(os.fspath(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != GL_OK:
        msg = load().gl_last_error().decode(errors="replace")
        raise GlaucisError(f"{what} failed (rc={rc}): {msg}")


def device_status(stream_ptr: int | None = None, err_word: int | None = None) -> int:
    """Synchronises the stream and returns (and clears) the device error word."""
    code = ctypes.c_int(0)
    check(load().gl_device_status(err_word, stream_ptr, ctypes.byref(code)), "gl_device_status")
    return code.value
