"""ctypes binding of libblackflash_b200.so (the C ABI in include/blackflash_b200.h).

There is no CPU or pure-PyTorch fallback: if the library is missing or cannot
be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

BF_OK, BF_ERR_ARG, BF_ERR_CUDA, BF_ERR_TIMEOUT = 0, 1, 2, 3

# Every symbol the header declares (checked by the CPU test suite).
EXPORTED = (
    "blackflash_fwd",
    "blackflash_fwd_causal",
    "blackflash_fwd_partial",
    "blackflash_fwd_partial_blocks",
    "blackflash_lse_merge",
    "blackflash_f32_to_bf16",
    "blackflash_bwd",
    "blackflash_bwd_workspace_bytes",
    "blackflash_bwd_noalloc",
    "blackflash_status",
    "blackflash_ring_create",
    "blackflash_ring_handle_bytes",
    "blackflash_ring_connect",
    "blackflash_ring_forward",
    "blackflash_ring_status",
    "blackflash_ring_destroy",
    "blackflash_fwd_timeout_probe",
    "blackflash_fwd_debug_s",
    "blackflash_fwd_trace",
    "blackflash_last_error",
    "blackflash_abi_version",
)

_lock = threading.Lock()
_lib = None

_vp, _fp, _i, _ll, _f = ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_longlong, ctypes.c_float

_SIGS = {
    "blackflash_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp]),
    "blackflash_fwd_causal": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp]),
    "blackflash_fwd_partial": (_i, [_vp, _vp, _vp, _vp, _vp, _ll, _i, _i, _i, _f, _vp]),
    "blackflash_fwd_partial_blocks": (_i, [_vp, _vp, _vp, _vp, _vp, _ll, _i, _i, _i, _i, _i, _f, _vp]),
    "blackflash_lse_merge": (_i, [_vp, _vp, _vp, _vp, _ll, _i, _vp]),
    "blackflash_bwd": (_i, [_vp] * 10 + [_ll, _i, _i, _i, _i, _f, _vp]),
    "blackflash_bwd_workspace_bytes": (_ll, [_i, _i, _i, _i]),
    "blackflash_bwd_noalloc": (_i, [_vp] * 9 + [_i, _i, _i, _i, _f, _vp]),
    "blackflash_f32_to_bf16": (_i, [_vp, _vp, _ll, _vp]),
    "blackflash_status": (_i, [_i, ctypes.POINTER(ctypes.c_uint)]),
    "blackflash_ring_create": (_i, [_i, _i, _ll, _i, _i, ctypes.POINTER(_vp), _vp]),
    "blackflash_ring_handle_bytes": (_i, []),
    "blackflash_ring_connect": (_i, [_vp, _vp]),
    "blackflash_ring_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _f, _vp]),
    "blackflash_ring_status": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_uint)]),
    "blackflash_ring_destroy": (_i, [_vp]),
    "blackflash_fwd_timeout_probe": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, ctypes.c_ulonglong, _vp]),
    "blackflash_fwd_debug_s": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp]),
    "blackflash_fwd_trace": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp]),
    "blackflash_last_error": (ctypes.c_char_p, []),
    "blackflash_abi_version": (_i, []),
}


def lib_path() -> str:
    return os.environ.get("BLACKFLASH_B200_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libblackflash_b200.so not found at {path}; build it with "
                    "`python -m blackflash_b200.build` (needs nvcc)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != BF_OK:
        msg = load().blackflash_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")
