"""Tensor-parallel entry point: all-reduce fused with residual add + RMSNorm + group quant.

In a tensor-parallel model the projection before the norm is row-parallel,
so every rank ends up with a partial sum of the activation and an all-reduce
normally runs before ``fused_add_rmsnorm_group_quant`` (the reference's
operator, src/task01_fused_add_rmsnorm_group_quant.py:1731). ``TPFusedNormQuant``
does both in one kernel per rank over NVLink peer memory: each rank reduces
its row slab of the partials (read from every rank with unicast bulk copies),
applies the operator and stores the outputs of its rows to every rank.

Buffers that peers read or write live in one symmetric-memory arena per rank
(``torch.distributed._symmetric_memory``): the partial input, the replicated
outputs and the kernel's signal words. The producer writes its partial into
``partial_buffer(M)``; after the call ``residual_out``, ``x_q``, ``x_scale``
(and ``norm_out``) views hold the full result on every rank.

Every rank must make the same sequence of calls with the same shapes; the
kernel's cross-rank waits are bounded (2 s) and report through ``status``.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_ALIGN = 256
_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16,
       torch.float32: _lib.DTYPE_FP32}
_Q = {torch.int8: _lib.DTYPE_INT8, torch.float8_e4m3fn: _lib.DTYPE_E4M3}
MAX_WORLD = 8
SIGNAL_WORDS = 2 * 1024 * 8


class FarqArArgs(ctypes.Structure):
    """Mirror of farq_ar_args_t (include/farq.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("x_dtype", ctypes.c_int32),
        ("gamma_dtype", ctypes.c_int32),
        ("norm_out_dtype", ctypes.c_int32),
        ("q_dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("epoch", ctypes.c_uint32),
        ("M", ctypes.c_int64),
        ("D", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("reserved0", ctypes.c_int32),
        ("partial", ctypes.c_void_p * MAX_WORLD),
        ("residual", ctypes.c_void_p),
        ("gamma", ctypes.c_void_p),
        ("residual_out", ctypes.c_void_p * MAX_WORLD),
        ("norm_out", ctypes.c_void_p * MAX_WORLD),
        ("x_q", ctypes.c_void_p * MAX_WORLD),
        ("x_scale", ctypes.c_void_p * MAX_WORLD),
        ("signal", ctypes.c_void_p * MAX_WORLD),
        ("status", ctypes.c_void_p),
    ]


def _up(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class TPFusedNormQuant:
    """Fused all-reduce + add + RMSNorm + group quant for one process group.

    Args:
      group: the tensor-parallel process group (default group if None).
      max_rows, hidden: largest M and the hidden size D.
      group_size, dtype, q_dtype: as for the single-GPU operator.
      norm_dtype: dtype of a replicated ``norm_out``; None skips it.
    """

    def __init__(self, max_rows: int, hidden: int, group_size: int = 128,
                 dtype: torch.dtype = torch.bfloat16,
                 q_dtype: torch.dtype = torch.float8_e4m3fn,
                 norm_dtype: torch.dtype | None = None, group=None,
                 device: torch.device | None = None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        if dtype not in (torch.bfloat16, torch.float16):
            raise TypeError(f"dtype {dtype} unsupported")
        if q_dtype not in _Q:
            raise TypeError(f"q_dtype {q_dtype} unsupported")
        if hidden % group_size:
            raise ValueError("hidden must be a multiple of group_size")
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > MAX_WORLD:
            raise ValueError(f"at most {MAX_WORLD} ranks")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.M, self.D, self.G = max_rows, hidden, group_size
        self.dtype, self.q_dtype, self.norm_dtype = dtype, q_dtype, norm_dtype
        es = torch.empty(0, dtype=dtype).element_size()
        ns = torch.empty(0, dtype=norm_dtype).element_size() if norm_dtype else 0
        N = max_rows * hidden
        off, layout = 0, {}
        for name, nbytes in (("partial", N * es), ("residual_out", N * es), ("norm_out", N * ns),
                             ("x_q", N), ("x_scale", max_rows * (hidden // group_size) * 4),
                             ("signal", SIGNAL_WORDS * 4)):
            layout[name] = off
            off += _up(nbytes)
        self._layout = layout
        # The kernel reads and writes peers with plain unicast accesses; the
        # arena is not bound to an NVLink multicast object (nothing here uses
        # multimem, and a rank that exits while its memory is bound to one
        # can fault the other ranks' GPUs).
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        self._arena = symm.empty(off, dtype=torch.uint8, device=self.device)
        self._arena[layout["signal"]: layout["signal"] + SIGNAL_WORDS * 4].zero_()
        torch.cuda.synchronize(self.device)
        self._handle = symm.rendezvous(self._arena, self.group.group_name)
        self._peers = [int(p) for p in self._handle.buffer_ptrs]
        self.epoch = 0
        # Per-call work is kept small: the argument struct with every peer
        # pointer is built once, only M, epoch, residual, gamma change.
        a = FarqArArgs()
        a.struct_size = ctypes.sizeof(FarqArArgs)
        a.x_dtype = _DT[self.dtype]
        a.norm_out_dtype = _DT[self.norm_dtype] if self.norm_dtype else 0
        a.q_dtype = _Q[self.q_dtype]
        a.group_size = self.G
        a.world = self.world
        a.rank = self.rank
        a.D = self.D
        L = self._layout
        for k, base in enumerate(self._peers):
            a.partial[k] = base + L["partial"]
            a.residual_out[k] = base + L["residual_out"]
            a.norm_out[k] = base + L["norm_out"] if self.norm_dtype else None
            a.x_q[k] = base + L["x_q"]
            a.x_scale[k] = base + L["x_scale"]
            a.signal[k] = base + L["signal"]
        self._args = a
        self._args_ref = ctypes.byref(a)
        self._views = {}
        self._lib = _lib.load()
        dist.barrier(group=self.group)

    def _view(self, name, dtype, shape):
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        o = self._layout[name]
        return self._arena[o:o + nbytes].view(dtype).view(*shape)

    def partial_buffer(self, M: int) -> torch.Tensor:
        """[M, D] view the producer writes this rank's partial activation into."""
        return self._view("partial", self.dtype, (self.M, self.D))[:M]

    def outputs(self, M: int):
        """(residual_out, norm_out or None, x_q, x_scale) views of the replicated outputs."""
        ro = self._view("residual_out", self.dtype, (self.M, self.D))[:M]
        no = (self._view("norm_out", self.norm_dtype, (self.M, self.D))[:M]
              if self.norm_dtype else None)
        q = self._view("x_q", torch.uint8, (self.M, self.D))[:M].view(self.q_dtype)
        s = self._view("x_scale", torch.float32, (self.M, self.D // self.G))[:M]
        return ro, no, q, s

    def __call__(self, M: int, residual: torch.Tensor, gamma: torch.Tensor, eps: float, *,
                 ue8m0: bool = False, status: torch.Tensor | None = None,
                 _test_force_timeout: bool = False, _fused_at_world1: bool = False):
        """x = sum over ranks of partial_buffer(M); returns the replicated
        (residual_out, norm_out, x_q, x_scale) of the operator on x."""
        if not 0 <= M <= self.M:
            raise ValueError(f"M={M} outside [0, {self.M}]")
        if residual.shape != (M, self.D) or residual.dtype != self.dtype or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous [M, D] tensor of the arena dtype")
        if residual.device != self.device or gamma.device != self.device:
            raise TypeError("residual and gamma must be on this rank's device")
        if gamma.shape != (self.D,) or gamma.dtype not in _DT:
            raise ValueError("gamma must be a [D] float tensor")
        self.epoch += 1
        a = self._args
        a.gamma_dtype = _DT[gamma.dtype]
        a.flags = ((_lib.FLAG_UE8M0 if ue8m0 else 0)
                   | (_lib.FLAG_TEST_FORCE_TIMEOUT if _test_force_timeout else 0)
                   | (_lib.FLAG_AR_KERNEL_AT_WORLD1 if _fused_at_world1 else 0))
        a.epoch = self.epoch & 0xFFFFFFFF
        a.M = M
        a.eps = float(eps)
        a.residual = residual.data_ptr()
        a.gamma = gamma.data_ptr()
        a.status = status.data_ptr() if status is not None else None
        st = self._lib.farq_ar_launch(self._args_ref,
                                      torch.cuda.current_stream(self.device).cuda_stream)
        if st != _lib.OK:
            raise RuntimeError(f"farq_ar_launch failed: {_lib.strerror(st)} (status {st})")
        out = self._views.get(M)
        if out is None:
            out = self._views[M] = self.outputs(M)
        return out
