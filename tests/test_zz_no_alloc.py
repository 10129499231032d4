"""The host-buffer entry point that allocates no device memory
(farq_launch_host_noalloc), called through the C ABI.

It exists for callers that hold their tensors in host memory and must not
allocate on the GPU themselves (a plugin inside a process whose device memory
is owned by another framework's allocator, or C/FFI code with host buffers
only): it stages every call through a fixed array compiled into libfarq.so.
Its outputs must equal those of the regular device entry point (farq_launch,
through fused_add_rmsnorm_group_quant) bit for bit — the same kernel computes
both — on consecutive calls that reuse the shared array.

This file is collected last on purpose, and is meant to pass both alone in a
fresh process and after every other test.
"""
import ctypes

import pytest
import torch

from flagos_kernelgen_72h_shanghai_2026_b200 import _lib, fused_add_rmsnorm_group_quant
from flagos_kernelgen_72h_shanghai_2026_b200.workloads import Workload, make_inputs

pytestmark = pytest.mark.gpu

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16,
       torch.float32: _lib.DTYPE_FP32}
_Q = {torch.int8: _lib.DTYPE_INT8, torch.float8_e4m3fn: _lib.DTYPE_E4M3}


def _host_call(x, r, g, ro, no, q, s, eps, G, ue8m0=False):
    lib = _lib.load()
    lib.farq_launch_host_noalloc.argtypes = [ctypes.POINTER(_lib.FarqArgs), ctypes.c_void_p]
    lib.farq_launch_host_noalloc.restype = ctypes.c_int
    a = _lib.FarqArgs()
    a.struct_size = ctypes.sizeof(a)
    a.x_dtype = _DT[x.dtype]
    a.gamma_dtype = _DT[g.dtype]
    a.residual_out_dtype = _DT[ro.dtype]
    a.norm_out_dtype = _DT[no.dtype] if no is not None else 0
    a.q_dtype = _Q[q.dtype]
    a.flags = _lib.FLAG_UE8M0 if ue8m0 else 0
    a.group_size = G
    a.M, a.D = x.shape
    a.eps = eps
    a.x, a.residual, a.gamma = x.data_ptr(), r.data_ptr(), g.data_ptr()
    a.residual_out = ro.data_ptr()
    a.norm_out = no.data_ptr() if no is not None else None
    a.x_q, a.x_scale = q.data_ptr(), s.data_ptr()
    stream = torch.cuda.current_stream()
    st = lib.farq_launch_host_noalloc(ctypes.byref(a), stream.cuda_stream)
    stream.synchronize()
    return st


def _device_call(x, r, g, ro_dtype, no_dtype, q_dtype, eps, G, ue8m0=False):
    M, D = x.shape
    xd, rd, gd = x.cuda(), r.cuda(), g.cuda()
    ro = torch.empty(M, D, dtype=ro_dtype, device="cuda")
    no = torch.empty(M, D, dtype=no_dtype, device="cuda") if no_dtype else None
    q = torch.empty(M, D, dtype=q_dtype, device="cuda")
    s = torch.empty(M, D // G, device="cuda")
    fused_add_rmsnorm_group_quant(xd, rd, gd, ro, no, q, s, eps, G, ue8m0=ue8m0)
    torch.cuda.synchronize()
    return ro.cpu(), None if no is None else no.cpu(), q.cpu(), s.cpu()


def _same(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def test_noalloc_entry_matches_device_entry_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    torch.cuda.set_device(0)
    cases = [  # (workload, norm_out dtype, pinned host memory)
        (Workload("na1", 700, 7168, res_std=2.0, seed=51), torch.bfloat16, True),
        (Workload("na2", 513, 5120, dtype=torch.float16, group_size=64, eps=1e-5,
                  q_dtype=torch.int8, seed=52), None, False),
    ]
    for w, no_dtype, pinned in cases:
        x, r, g = make_inputs(w)
        M, D, G = w.M, w.D, w.group_size
        ref = _device_call(x, r, g, x.dtype, no_dtype, w.q_dtype, w.eps, G)
        ro = torch.empty(M, D, dtype=x.dtype)
        no = torch.empty(M, D, dtype=no_dtype) if no_dtype else None
        q = torch.empty(M, D, dtype=w.q_dtype)
        s = torch.empty(M, D // G)
        if pinned:
            x, r, g = x.pin_memory(), r.pin_memory(), g.pin_memory()
            ro, q, s = ro.pin_memory(), q.pin_memory(), s.pin_memory()
            no = no.pin_memory() if no is not None else None
        assert _host_call(x, r, g, ro, no, q, s, w.eps, G) == _lib.OK
        assert _same(ro, ref[0]) and _same(q, ref[2]) and _same(s, ref[3])
        if no is not None:
            assert _same(no, ref[1])


def test_noalloc_entry_rejects_calls_beyond_its_array():
    lib = _lib.load()
    w = Workload("big", 2000, 7168)  # ~100 MB of staging > 64 MiB
    x = torch.zeros(w.M, w.D, dtype=torch.bfloat16)
    g = torch.ones(w.D, dtype=torch.bfloat16)
    ro = torch.empty_like(x)
    q = torch.empty(w.M, w.D, dtype=torch.float8_e4m3fn)
    s = torch.empty(w.M, w.groups)
    assert _host_call(x, x, g, ro, None, q, s, w.eps, 128) == _lib.ERR_NOALLOC_TOO_LARGE
    assert b"64 MiB" in lib.farq_strerror(_lib.ERR_NOALLOC_TOO_LARGE)
