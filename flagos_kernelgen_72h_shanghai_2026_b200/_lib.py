"""ctypes binding of libfarq.so (C ABI: include/farq.h).

Loading fails loudly: there is no CPU or eager-PyTorch fallback behind this
module. If the library is missing, build it with
``python -m flagos_kernelgen_72h_shanghai_2026_b200._build``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from ._build import LIB_PATH

# enum farq_dtype
DTYPE_BF16, DTYPE_FP16, DTYPE_FP32, DTYPE_INT8, DTYPE_E4M3 = 0, 1, 2, 3, 4
FLAG_UE8M0 = 1
FLAG_SCALE_COLUMN_MAJOR = 2
FLAG_AR_KERNEL_AT_WORLD1 = 4
FLAG_TEST_FORCE_TIMEOUT = 1 << 30  # test only, see include/farq.h

# enum farq_status
OK = 0
ERR_NULL_POINTER = 1
ERR_BAD_SHAPE = 2
ERR_BAD_GROUP = 3
ERR_BAD_DTYPE = 4
ERR_ALIGNMENT = 5
ERR_UNSUPPORTED = 6
ERR_CUDA = 7
ERR_BAD_ARGS_SIZE = 8
ERR_DEVICE_TIMEOUT = 9
ERR_NOALLOC_TOO_LARGE = 10

ABI_VERSION = 1


class FarqArgs(ctypes.Structure):
    """Mirror of farq_args_t (field order and types must match include/farq.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("x_dtype", ctypes.c_int32),
        ("gamma_dtype", ctypes.c_int32),
        ("residual_out_dtype", ctypes.c_int32),
        ("norm_out_dtype", ctypes.c_int32),
        ("q_dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("M", ctypes.c_int64),
        ("D", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("tune_ctas_per_sm", ctypes.c_int32),
        ("tune_teams_per_cta", ctypes.c_int32),
        ("tune_stages", ctypes.c_int32),
        ("tune_vec_per_thread", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("gamma", ctypes.c_void_p),
        ("residual_out", ctypes.c_void_p),
        ("norm_out", ctypes.c_void_p),
        ("x_q", ctypes.c_void_p),
        ("x_scale", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("x_row_stride", ctypes.c_int64),
        ("residual_row_stride", ctypes.c_int64),
        ("residual_out_row_stride", ctypes.c_int64),
        ("norm_out_row_stride", ctypes.c_int64),
        ("x_q_row_stride", ctypes.c_int64),
        ("x_scale_row_stride", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libfarq.so once and declare its prototypes. Raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libfarq.so not found at {p}; the CUDA path has no fallback. "
                "Build it with: python -m flagos_kernelgen_72h_shanghai_2026_b200._build"
            )
        lib = ctypes.CDLL(str(p))
        lib.farq_launch.argtypes = [ctypes.POINTER(FarqArgs), ctypes.c_void_p]
        lib.farq_launch.restype = ctypes.c_int
        lib.farq_strerror.argtypes = [ctypes.c_int]
        lib.farq_strerror.restype = ctypes.c_char_p
        lib.farq_abi_version.argtypes = []
        lib.farq_abi_version.restype = ctypes.c_int
        lib.farq_max_hidden.argtypes = []
        lib.farq_max_hidden.restype = ctypes.c_int64
        lib.farq_plan.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.POINTER(ctypes.c_int64)]
        lib.farq_plan.restype = ctypes.c_int
        lib.farq_ar_launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.farq_ar_launch.restype = ctypes.c_int
        v = lib.farq_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"libfarq.so ABI version {v} != expected {ABI_VERSION}; rebuild it")
        if path is None:
            _lib = lib
        return lib


def strerror(status: int) -> str:
    return load().farq_strerror(status).decode()


def plan(M: int, D: int, group_size: int, x_dtype: int, ctas_per_sm: int = 0, teams: int = 0,
         stages: int = 0, vec_per_thread: int = 0) -> dict:
    """The launch plan farq_launch would use on the current device."""
    out = (ctypes.c_int64 * 6)()
    st = load().farq_plan(M, D, group_size, x_dtype, ctas_per_sm, teams, stages, vec_per_thread,
                          out)
    if st != OK:
        raise RuntimeError(f"farq_plan: {strerror(st)}")
    return dict(team_threads=out[0], teams=out[1], vec_per_thread=out[2], grid=out[3],
                stages=out[4], smem=out[5])
