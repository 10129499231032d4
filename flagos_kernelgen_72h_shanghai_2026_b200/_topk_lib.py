"""ctypes binding of libdsa_topk.so (C ABI: include/dsa_topk.h).

Loading fails loudly: there is no CPU or eager-PyTorch fallback behind this
module. If the library is missing, build it with
``python -m flagos_kernelgen_72h_shanghai_2026_b200._build``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from ._build import TOPK_LIB_PATH

# enum dsa_topk_dtype
DTYPE_FP32, DTYPE_BF16, DTYPE_FP16, DTYPE_INT32, DTYPE_INT64 = 0, 1, 2, 3, 4

# enum dsa_topk_status
OK = 0
ERR_NULL_POINTER = 1
ERR_BAD_SHAPE = 2
ERR_BAD_TOPK = 3
ERR_BAD_DTYPE = 4
ERR_ALIGNMENT = 5
ERR_UNSUPPORTED = 6
ERR_CUDA = 7
ERR_BAD_ARGS_SIZE = 8

ABI_VERSION = 1
MAX_BLOCKS = 16384
MAX_TOPK = 2048


class DsaTopkArgs(ctypes.Structure):
    """Mirror of dsa_topk_args_t (field order and types must match include/dsa_topk.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("scores_dtype", ctypes.c_int32),
        ("index_dtype", ctypes.c_int32),
        ("page_dtype", ctypes.c_int32),
        ("blocks_dtype", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("B", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("Q", ctypes.c_int64),
        ("NB", ctypes.c_int64),
        ("scores", ctypes.c_void_p),
        ("page_table", ctypes.c_void_p),
        ("q_pos", ctypes.c_void_p),
        ("kv_lens", ctypes.c_void_p),
        ("out_blocks", ctypes.c_void_p),
        ("out_pages", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libdsa_topk.so once and declare its prototypes. Raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else TOPK_LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libdsa_topk.so not found at {p}; the CUDA path has no fallback. "
                "Build it with: python -m flagos_kernelgen_72h_shanghai_2026_b200._build"
            )
        lib = ctypes.CDLL(str(p))
        lib.dsa_topk_launch.argtypes = [ctypes.POINTER(DsaTopkArgs), ctypes.c_void_p]
        lib.dsa_topk_launch.restype = ctypes.c_int
        lib.dsa_topk_strerror.argtypes = [ctypes.c_int]
        lib.dsa_topk_strerror.restype = ctypes.c_char_p
        lib.dsa_topk_abi_version.argtypes = []
        lib.dsa_topk_abi_version.restype = ctypes.c_int
        v = lib.dsa_topk_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"libdsa_topk.so ABI version {v} != expected {ABI_VERSION}; rebuild it")
        if path is None:
            _lib = lib
        return lib


def strerror(status: int) -> str:
    return load().dsa_topk_strerror(status).decode()
