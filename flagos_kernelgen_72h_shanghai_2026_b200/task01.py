"""Host-side mirror of the reference operator for Task 01.

``fused_add_rmsnorm_group_quant`` keeps the competition signature of
src/task01_fused_add_rmsnorm_group_quant.py:1731-1741 (x, residual, gamma,
residual_out, norm_out, x_q, x_scale, eps, group_size), writes into the
caller's tensors and returns the same four objects (:1790, :1817, :1728).

What the reference routes by backend tag and (M, D) (:1744-1851) is one
kernel here; the host only validates and fills the C-ABI argument struct.

Extensions over the reference, all keyword-or-type driven so positional
callers see the reference contract:
  * ``x_q.dtype``: ``torch.int8`` gives the reference semantics (scale over
    127, clamp, truncation toward zero, :1089-1104); ``torch.float8_e4m3fn``
    gives scale over 448 and a saturating round-to-nearest-even cast.
  * ``norm_out`` may be ``None`` or empty: the normalised tensor is skipped.
  * ``ue8m0=True`` rounds every scale up to a power of two.
  * Row-strided (inner-contiguous) views are accepted, and ``x_scale`` may be
    a column-major view (``buf[:, :M].t()`` of a ``[D/G, ld]`` buffer), the
    scale layout blockwise-FP8 GEMMs read.

Errors: ``TypeError`` for a non-CUDA tensor or a dtype the kernel does not
take, ``ValueError`` for shapes, group sizes and alignment, ``RuntimeError``
when a CUDA call fails. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

try:  # C++ launch path (csrc/farq_fast.cpp); without it every call takes the ctypes path
    from . import _farq_fast as _fast
except ImportError:
    _fast = None
_T = torch.Tensor

_IN_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16}
_FLOAT_DTYPES = {
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float16: _lib.DTYPE_FP16,
    torch.float32: _lib.DTYPE_FP32,
}
_Q_DTYPES = {torch.int8: _lib.DTYPE_INT8, torch.float8_e4m3fn: _lib.DTYPE_E4M3}
_ARGS_SIZE = ctypes.sizeof(_lib.FarqArgs)

_VALUE_ERRORS = {
    _lib.ERR_BAD_SHAPE,
    _lib.ERR_BAD_GROUP,
    _lib.ERR_ALIGNMENT,
    _lib.ERR_UNSUPPORTED,
    _lib.ERR_NULL_POINTER,
}


def _check_cuda(name: str, t: torch.Tensor, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device != device:
        raise TypeError(f"{name} is on {t.device}, expected {device} (CUDA tensors only)")


def _row_stride(name: str, t: torch.Tensor, rows: int, cols: int) -> int:
    if t.dim() != 2 or t.shape[0] != rows or t.shape[1] != cols:
        raise ValueError(f"{name} must have shape [{rows}, {cols}], got {list(t.shape)}")
    if cols > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must be contiguous along its last dimension")
    return t.stride(0) if rows > 1 else cols


# Per-thread cache of filled argument structs keyed by every piece of tensor
# metadata the Python checks read (device, shape, strides, dtype of each
# tensor) and the scalar arguments. A hit skips the Python-side checks and
# the struct fill: only the data pointers change. farq_launch still validates
# every call (alignment of the new pointers included).
_tls = threading.local()
_CACHE_MAX = 64


def _meta(t):
    return (t.device, t.shape, t.stride(), t.dtype)


def _raise_status(st: int):
    msg = f"farq_launch failed: {_lib.strerror(st)} (status {st})"
    if st in _VALUE_ERRORS:
        raise ValueError(msg)
    if st == _lib.ERR_BAD_DTYPE:
        raise TypeError(msg)
    raise RuntimeError(msg)


def _launch(a, device):
    lib = _lib.load()
    if torch.cuda.current_device() != device.index:
        with torch.cuda.device(device):
            st = lib.farq_launch(ctypes.byref(a), torch.cuda.current_stream(device).cuda_stream)
    else:
        st = lib.farq_launch(ctypes.byref(a), torch.cuda.current_stream(device).cuda_stream)
    if st != _lib.OK:
        _raise_status(st)


def fused_add_rmsnorm_group_quant(
    x: torch.Tensor,
    residual: torch.Tensor,
    gamma: torch.Tensor,
    residual_out: torch.Tensor,
    norm_out: torch.Tensor | None,
    x_q: torch.Tensor,
    x_scale: torch.Tensor,
    eps: float,
    group_size: int,
    *,
    ue8m0: bool = False,
    _tune_ctas_per_sm: int = 0,
    _tune_teams_per_cta: int = 0,
    _tune_stages: int = 0,
    _tune_vec_per_thread: int = 0,
    _status: torch.Tensor | None = None,
    _test_force_timeout: bool = False,
):
    """residual_out = x + residual; norm = RMSNorm(residual_out) * gamma;
    per-group quantisation of norm into (x_q, x_scale). Asynchronous on the
    current CUDA stream; returns (residual_out, norm_out, x_q, x_scale)."""
    # C++ launch path for the common case (contiguous tensors on one device,
    # no test or tuning options); -1 = not handled, continue below.
    if (_fast is not None and _T is type(x) and _T is type(residual) and _T is type(gamma)
            and _T is type(residual_out) and _T is type(x_q) and _T is type(x_scale)
            and (norm_out is None or _T is type(norm_out)) and _status is None
            and not (_test_force_timeout or _tune_ctas_per_sm or _tune_teams_per_cta
                     or _tune_stages or _tune_vec_per_thread)):
        try:
            st = _fast.task01(x, residual, gamma, residual_out, norm_out, x_q, x_scale, eps,
                              group_size, bool(ue8m0))
        except TypeError:  # a scalar pybind11 cannot convert: the checks below report it
            st = -1
        if st == _lib.OK:
            return residual_out, norm_out, x_q, x_scale
        if st > 0:
            _raise_status(st)
    key = None
    if (isinstance(x, torch.Tensor) and isinstance(residual, torch.Tensor)
            and isinstance(gamma, torch.Tensor) and isinstance(residual_out, torch.Tensor)
            and isinstance(x_q, torch.Tensor) and isinstance(x_scale, torch.Tensor)
            and (norm_out is None or isinstance(norm_out, torch.Tensor))):
        key = (_meta(x), _meta(residual), _meta(gamma), _meta(residual_out),
               None if norm_out is None else _meta(norm_out), _meta(x_q), _meta(x_scale),
               eps, group_size, ue8m0, _tune_ctas_per_sm, _tune_teams_per_cta, _tune_stages,
               _tune_vec_per_thread, _status is None, _test_force_timeout)
        cache = getattr(_tls, "args", None)
        a = cache.get(key) if cache is not None else None
        if a is not None:
            a.x = x.data_ptr()
            a.residual = residual.data_ptr()
            a.gamma = gamma.data_ptr()
            a.residual_out = residual_out.data_ptr()
            a.norm_out = norm_out.data_ptr() if a.norm_out else None
            a.x_q = x_q.data_ptr()
            a.x_scale = x_scale.data_ptr()
            a.status = _status.data_ptr() if _status is not None else None
            _launch(a, x.device)
            return residual_out, norm_out, x_q, x_scale
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
    device = x.device
    if device.type != "cuda":
        raise TypeError(f"x is on {device}; this operator runs on CUDA devices only")
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, D], got shape {list(x.shape)}")
    M, D = x.shape
    for name, t in (("residual", residual), ("gamma", gamma), ("residual_out", residual_out),
                    ("x_q", x_q), ("x_scale", x_scale)):
        _check_cuda(name, t, device)
    write_norm = norm_out is not None and norm_out.numel() > 0
    if write_norm:
        _check_cuda("norm_out", norm_out, device)

    x_dt = _IN_DTYPES.get(x.dtype)
    if x_dt is None:
        raise TypeError(f"x dtype {x.dtype} unsupported (bfloat16 or float16)")
    if residual.dtype != x.dtype:
        raise TypeError(f"residual dtype {residual.dtype} must equal x dtype {x.dtype}")
    g_dt = _FLOAT_DTYPES.get(gamma.dtype)
    ro_dt = _FLOAT_DTYPES.get(residual_out.dtype)
    q_dt = _Q_DTYPES.get(x_q.dtype)
    if g_dt is None:
        raise TypeError(f"gamma dtype {gamma.dtype} unsupported")
    if ro_dt is None:
        raise TypeError(f"residual_out dtype {residual_out.dtype} unsupported")
    if q_dt is None:
        raise TypeError(f"x_q dtype {x_q.dtype} unsupported (int8 or float8_e4m3fn)")
    if x_scale.dtype != torch.float32:
        raise TypeError(f"x_scale dtype {x_scale.dtype} must be float32")
    no_dt = 0
    if write_norm:
        no_dt = _FLOAT_DTYPES.get(norm_out.dtype)
        if no_dt is None:
            raise TypeError(f"norm_out dtype {norm_out.dtype} unsupported")

    group_size = int(group_size)
    if group_size <= 0 or D % group_size != 0:
        raise ValueError(f"hidden size {D} is not a multiple of group_size {group_size}")
    if gamma.dim() != 1 or gamma.shape[0] != D or (D > 1 and gamma.stride(0) != 1):
        raise ValueError(f"gamma must be a contiguous [{D}] vector, got {list(gamma.shape)}")
    groups = D // group_size
    sx = _row_stride("x", x, M, D)
    sr = _row_stride("residual", residual, M, D)
    sro = _row_stride("residual_out", residual_out, M, D)
    sq = _row_stride("x_q", x_q, M, D)
    # x_scale may be a column-major ("MN-major") view, e.g. buf[:, :M].t() of a
    # [groups, ld] buffer as blockwise-FP8 GEMMs take it.
    scale_cm = (x_scale.dim() == 2 and tuple(x_scale.shape) == (M, groups) and M > 1
                and x_scale.stride(0) == 1 and x_scale.stride(1) >= M and groups > 1)
    ss = x_scale.stride(1) if scale_cm else _row_stride("x_scale", x_scale, M, groups)
    sno = _row_stride("norm_out", norm_out, M, D) if write_norm else 0
    if M == 0:
        return residual_out, norm_out, x_q, x_scale

    a = _lib.FarqArgs()
    a.struct_size = _ARGS_SIZE
    a.x_dtype = x_dt
    a.gamma_dtype = g_dt
    a.residual_out_dtype = ro_dt
    a.norm_out_dtype = no_dt
    a.q_dtype = q_dt
    a.flags = (_lib.FLAG_UE8M0 if ue8m0 else 0) | (
        _lib.FLAG_SCALE_COLUMN_MAJOR if scale_cm else 0) | (
        _lib.FLAG_TEST_FORCE_TIMEOUT if _test_force_timeout else 0)
    a.group_size = group_size
    a.M = M
    a.D = D
    a.eps = float(eps)
    a.tune_ctas_per_sm = int(_tune_ctas_per_sm)
    a.tune_teams_per_cta = int(_tune_teams_per_cta)
    a.tune_stages = int(_tune_stages)
    a.tune_vec_per_thread = int(_tune_vec_per_thread)
    a.x = x.data_ptr()
    a.residual = residual.data_ptr()
    a.gamma = gamma.data_ptr()
    a.residual_out = residual_out.data_ptr()
    a.norm_out = norm_out.data_ptr() if write_norm else None
    a.x_q = x_q.data_ptr()
    a.x_scale = x_scale.data_ptr()
    a.status = _status.data_ptr() if _status is not None else None
    a.x_row_stride = sx
    a.residual_row_stride = sr
    a.residual_out_row_stride = sro
    a.norm_out_row_stride = sno
    a.x_q_row_stride = sq
    a.x_scale_row_stride = ss

    _launch(a, device)
    if key is not None:
        cache = getattr(_tls, "args", None)
        if cache is None:
            cache = _tls.args = {}
        if len(cache) >= _CACHE_MAX:
            cache.pop(next(iter(cache)))
        cache[key] = a
    return residual_out, norm_out, x_q, x_scale


def launch_plan(M: int, D: int, group_size: int = 128, dtype: torch.dtype = torch.bfloat16,
                ctas_per_sm: int = 0, teams: int = 0, stages: int = 0,
                vec_per_thread: int = 0) -> dict:
    """Launch plan (team threads, teams per CTA, vectors per thread, grid,
    slots per team, shared-memory bytes) on the current device."""
    return _lib.plan(M, D, group_size, _IN_DTYPES[dtype], ctas_per_sm, teams, stages,
                     vec_per_thread)
