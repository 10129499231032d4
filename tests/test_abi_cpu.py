"""The C-ABI library loads and exports every entry point include/farq.h
declares; argument validation answers with status codes before any device
work (runs without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from flagos_kernelgen_72h_shanghai_2026_b200 import _lib
from flagos_kernelgen_72h_shanghai_2026_b200._build import LIB_PATH, build_lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "farq.h"


@pytest.fixture(scope="module")
def lib():
    build_lib()
    return _lib.load()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(farq_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"farq_launch", "farq_strerror", "farq_abi_version", "farq_max_hidden",
            "farq_plan", "farq_ar_launch"} <= set(names)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(LIB_PATH))
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} declared in farq.h but not exported"


def test_struct_layout_matches_header(lib):
    # The header's farq_args_t: 8 x 4-byte fields, 2 x int64, 6 x 4-byte, 8 pointers, 6 int64
    assert ctypes.sizeof(_lib.FarqArgs) == 8 * 4 + 2 * 8 + 6 * 4 + 8 * 8 + 6 * 8
    a = _lib.FarqArgs()
    a.struct_size = ctypes.sizeof(a) + 8
    assert lib.farq_launch(ctypes.byref(a), None) == _lib.ERR_BAD_ARGS_SIZE


def test_reserved_field_must_be_zero(lib):
    a = _args(reserved0=1)
    assert lib.farq_launch(ctypes.byref(a), None) == _lib.ERR_BAD_ARGS_SIZE


def test_version_and_limits(lib):
    assert lib.farq_abi_version() == _lib.ABI_VERSION
    assert lib.farq_max_hidden() == 16384
    for code in range(0, 10):
        assert lib.farq_strerror(code)
    assert b"unknown" in lib.farq_strerror(1234)


def _args(**kw):
    a = _lib.FarqArgs()
    a.struct_size = ctypes.sizeof(a)
    a.x_dtype = _lib.DTYPE_BF16
    a.gamma_dtype = _lib.DTYPE_BF16
    a.residual_out_dtype = _lib.DTYPE_BF16
    a.norm_out_dtype = _lib.DTYPE_BF16
    a.q_dtype = _lib.DTYPE_E4M3
    a.group_size = 128
    a.M, a.D, a.eps = 4, 1024, 1e-6
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    (dict(group_size=96), _lib.ERR_BAD_GROUP),
    (dict(group_size=4), _lib.ERR_BAD_GROUP),
    (dict(group_size=512), _lib.ERR_BAD_GROUP),
    (dict(D=1000), _lib.ERR_BAD_SHAPE),
    (dict(D=1024 + 64, group_size=128), _lib.ERR_BAD_SHAPE),
    (dict(M=-1), _lib.ERR_BAD_SHAPE),
    (dict(D=32768), _lib.ERR_UNSUPPORTED),
    (dict(x_dtype=_lib.DTYPE_FP32), _lib.ERR_BAD_DTYPE),
    (dict(q_dtype=_lib.DTYPE_BF16), _lib.ERR_BAD_DTYPE),
    (dict(gamma_dtype=_lib.DTYPE_INT8), _lib.ERR_BAD_DTYPE),
    (dict(), _lib.ERR_NULL_POINTER),
])
def test_validation_codes(lib, kw, code):
    assert lib.farq_launch(ctypes.byref(_args(**kw)), None) == code


def test_m_zero_is_a_noop(lib):
    assert lib.farq_launch(ctypes.byref(_args(M=0)), None) == _lib.OK


def test_misaligned_pointer_rejected(lib):
    a = _args(x=0x1008, residual=0x2000, gamma=0x3000, residual_out=0x4000,
              x_q=0x5000, x_scale=0x6000)
    assert lib.farq_launch(ctypes.byref(a), None) == _lib.ERR_ALIGNMENT
    a = _args(x=0x1000, residual=0x2000, gamma=0x3000, residual_out=0x4000,
              x_q=0x5000, x_scale=0x6000, x_row_stride=1028)
    assert lib.farq_launch(ctypes.byref(a), None) == _lib.ERR_ALIGNMENT


def test_null_args_pointer(lib):
    assert lib.farq_launch(None, None) == _lib.ERR_NULL_POINTER


def test_python_wrapper_refuses_cpu_tensors():
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="CUDA"):
        fused_add_rmsnorm_group_quant(x, x, torch.ones(256, dtype=torch.bfloat16), x.clone(), None,
                                      torch.zeros(2, 256, dtype=torch.int8),
                                      torch.zeros(2, 2), 1e-6, 128)


def test_ar_entry_validation_codes(lib):
    from flagos_kernelgen_72h_shanghai_2026_b200.tp import FarqArArgs
    a = FarqArArgs()
    a.struct_size = ctypes.sizeof(a) + 4
    assert lib.farq_ar_launch(ctypes.byref(a), None) == _lib.ERR_BAD_ARGS_SIZE
    a = FarqArArgs()
    a.struct_size = ctypes.sizeof(a)
    a.x_dtype, a.gamma_dtype, a.q_dtype, a.group_size = _lib.DTYPE_BF16, _lib.DTYPE_BF16, _lib.DTYPE_E4M3, 128
    a.M, a.D, a.world, a.rank = 8, 1024, 2, 2
    assert lib.farq_ar_launch(ctypes.byref(a), None) == _lib.ERR_BAD_SHAPE  # rank >= world
    a.rank, a.world = 0, 9
    assert lib.farq_ar_launch(ctypes.byref(a), None) == _lib.ERR_BAD_SHAPE  # world > 8
    a.world = 2
    assert lib.farq_ar_launch(ctypes.byref(a), None) == _lib.ERR_NULL_POINTER
    a.M = 0
    assert lib.farq_ar_launch(ctypes.byref(a), None) == _lib.OK


def test_noalloc_entry_validation_before_any_device_call(lib):
    f = lib.farq_launch_host_noalloc
    f.argtypes = [ctypes.POINTER(_lib.FarqArgs), ctypes.c_void_p]
    f.restype = ctypes.c_int
    assert f(None, None) == _lib.ERR_NULL_POINTER
    a = _args(struct_size=4)
    assert f(ctypes.byref(a), None) == _lib.ERR_BAD_ARGS_SIZE
    assert f(ctypes.byref(_args(group_size=100)), None) == _lib.ERR_BAD_GROUP
    assert f(ctypes.byref(_args(x_row_stride=2048)), None) == _lib.ERR_BAD_SHAPE  # host tensors contiguous
    assert f(ctypes.byref(_args()), None) == _lib.ERR_NULL_POINTER
    # 100k rows x 7168 needs far more than the 64 MiB staging array: rejected up front
    big = _args(M=100000, D=7168, x=0x1000, residual=0x2000, gamma=0x3000, residual_out=0x4000,
                x_q=0x5000, x_scale=0x6000)
    assert f(ctypes.byref(big), None) == _lib.ERR_NOALLOC_TOO_LARGE
    assert f(ctypes.byref(_args(M=0)), None) == _lib.OK


_HOST_PTRS = dict(x=0x1000, residual=0x2000, gamma=0x3000, residual_out=0x4000, x_q=0x5000,
                  x_scale=0x6000)


@pytest.mark.parametrize("kw,code", [
    # every check farq_launch makes on the arguments themselves comes before
    # the first copy: non-NULL (never dereferenced) host pointers prove that
    # no copy was queued, since queuing one from these addresses would fail
    # with a CUDA error instead of the validation code
    (dict(group_size=48, D=4800), _lib.ERR_BAD_GROUP),
    (dict(x_dtype=_lib.DTYPE_FP32), _lib.ERR_BAD_DTYPE),
    (dict(q_dtype=_lib.DTYPE_FP16), _lib.ERR_BAD_DTYPE),
    (dict(residual_out_dtype=_lib.DTYPE_INT8), _lib.ERR_BAD_DTYPE),
    (dict(norm_out=0x7000, norm_out_dtype=_lib.DTYPE_E4M3), _lib.ERR_BAD_DTYPE),
    (dict(reserved0=1), _lib.ERR_BAD_ARGS_SIZE),
    (dict(D=32768), _lib.ERR_UNSUPPORTED),
    (dict(M=-3), _lib.ERR_BAD_SHAPE),
    # M = 2^51 at D = 16384, G = 8 with fp32 residual_out: every staging term
    # is a multiple of 2^64 bytes, so an unchecked size sum wraps to a few KiB
    (dict(M=1 << 51, D=16384, group_size=8, residual_out_dtype=_lib.DTYPE_FP32),
     _lib.ERR_NOALLOC_TOO_LARGE),
    (dict(M=(64 << 20) // 1024 + 1), _lib.ERR_NOALLOC_TOO_LARGE),
])
def test_noalloc_entry_rejects_before_queuing_copies(lib, kw, code):
    f = lib.farq_launch_host_noalloc
    f.argtypes = [ctypes.POINTER(_lib.FarqArgs), ctypes.c_void_p]
    f.restype = ctypes.c_int
    a = _args(**{**_HOST_PTRS, **kw})
    assert f(ctypes.byref(a), None) == code
