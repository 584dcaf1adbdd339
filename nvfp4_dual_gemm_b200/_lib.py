"""ctypes binding of the C ABI in ``include/nvfp4_dual_gemm.h``.

The shared library is built in-tree (``nvfp4_dual_gemm_b200/libnvfp4dg.so``)
by ``nvfp4_dual_gemm_b200.build``.  There is no fallback: if the library is
missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                        "libnvfp4dg.so")

# Status codes (include/nvfp4_dual_gemm.h).
OK = 0
ERR_INVALID = 1
ERR_ALIGN = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE = 5
ERR_UNSUPPORTED = 6

# Flags.
FLAG_GRID_MASK = 0xFFF
FLAG_BN64 = 1 << 12
FLAG_BN128 = 1 << 13
FLAG_NO_STREAMK = 1 << 14
FLAG_SYNC_CHECK = 1 << 15
FLAG_FORCE_STREAMK = 1 << 17
FLAG_PAIR = 1 << 18
FLAG_NO_PAIR = 1 << 19
FLAG_SPLITK = 1 << 20
FLAG_NO_SPLITK = 1 << 21
FLAG_NO_PDL = 1 << 22
FLAG_NO_MERGED_B = 1 << 23
FLAG_STATIC_WEIGHTS = 1 << 24
FLAG_TEST_SK_TIMEOUT = 1 << 25
FLAG_NO_TMA_STORE = 1 << 26

# Input element types of nvfp4_quantize_rows.
DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

# Most weight slabs nvfp4_dual_gemm_run_host uses.
MAX_HOST_SLABS = 16

# Size of the static scratch behind nvfp4_dual_gemm_run_noalloc.
NOALLOC_SCRATCH_BYTES = 4 << 20

# Every symbol the header declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i = ctypes.c_int
_u = ctypes.c_uint
_sz = ctypes.c_size_t
_ip = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "nvfp4_dual_gemm_run": (_i, [_vp] * 7 + [_i, _i, _i, _i, _u, _vp]),
    "nvfp4_dual_gemm_workspace_size": (_sz, [_i, _i, _i, _i, _u]),
    "nvfp4_dual_gemm_run_ws": (_i, [_vp] * 7 + [_i, _i, _i, _i, _u, _vp, _sz,
                                                _vp]),
    "nvfp4_dual_gemm_run_noalloc": (_i, [_vp] * 7 + [_i, _i, _i, _i, _u,
                                                     _vp]),
    "nvfp4_dual_gemm_run_nvfp4_out": (_i, [_vp] * 8 + [_i, _i, _i, _i, _u,
                                                       _vp]),
    "nvfp4_dual_gemm_run_grouped": (_i, [_vp] * 7 + [_ip, _ip, _i, _i, _i,
                                                     _u, _vp, _sz, _vp]),
    "nvfp4_dual_gemm_grouped_workspace_size": (_sz, [_ip, _i, _i, _i, _u]),
    "nvfp4_quantize": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "nvfp4_quantize_rows": (_i, [_vp, _i, _i, _i, ctypes.c_longlong, _vp, _vp,
                                 _vp, _vp]),
    "nvfp4_scales_to_blocked": (_i, [_vp, _i, _i, ctypes.c_longlong, _vp,
                                     _vp]),
    "nvfp4_scales_from_blocked": (_i, [_vp, _i, _i, _vp, ctypes.c_longlong,
                                       _vp]),
    "nvfp4_dual_gemm_device_status": (_i, [_i, ctypes.POINTER(ctypes.c_uint)]),
    "nvfp4_dual_gemm_plan": (_i, [_i, _i, _i, _u, _i, _ip, _ip, _ip, _ip,
                                  _ip, _ip]),
    "nvfp4_dual_gemm_plan_work": (_i, [_i, _i, _i, _u, _i, _i, _ip, _i]),
    "nvfp4_dual_gemm_host_staging_size": (_sz, [_i, _i, _i, _i]),
    "nvfp4_dual_gemm_host_slabs": (_i, [_i, _i, _i, _i]),
    "nvfp4_dual_gemm_run_host": (_i, [_vp] * 7 + [_i, _i, _i, _i, _u, _i, _vp,
                                                  _sz, _vp]),
    "nvfp4_dual_gemm_last_error": (ctypes.c_char_p, []),
    "nvfp4_dual_gemm_version": (_i, []),
}

_lock = threading.Lock()
_lib = None


class NativeLibraryError(RuntimeError):
    """The CUDA library could not be loaded (no fallback exists)."""


def load() -> ctypes.CDLL:
    """Load libnvfp4dg.so (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryError(
                f"{LIB_PATH} is missing; build it with "
                "`python -m nvfp4_dual_gemm_b200.build`")
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as exc:  # pragma: no cover - depends on the machine
            raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


_ext_mod = None


def ext():
    """The torch binding ``_C`` (custom_kernel / cuda_nvfp4_dual_gemm /
    dual_gemm over the C ABI, built in-tree beside libnvfp4dg.so)."""
    global _ext_mod
    if _ext_mod is not None:
        return _ext_mod
    load()  # the binding links against the library loaded here
    try:
        from . import _C
    except ImportError as exc:
        raise NativeLibraryError(
            f"the torch binding _C is missing or fails to load ({exc}); "
            "build it with `python -m nvfp4_dual_gemm_b200.build`") from exc
    _ext_mod = _C
    return _C


def last_error() -> str:
    msg = load().nvfp4_dual_gemm_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Raise the Python exception matching a non-zero status code."""
    if rc == OK:
        return
    msg = f"{what} failed (status {rc}): {last_error()}"
    if rc in (ERR_INVALID, ERR_ALIGN, ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)
