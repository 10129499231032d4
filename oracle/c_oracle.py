"""ctypes wrapper of the plain-C restatement (oracle/farq_oracle.c).

TEST INFRASTRUCTURE / CPU BASELINE ONLY: imported by tests/ (cross-check of
oracle/farq_oracle.py) and by bench.py's CPU-baseline legs, never by the
product path. ``build()`` compiles it with gcc into oracle/_build/.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SRC = HERE / "farq_oracle.c"
LIB = HERE / "_build" / "libfarq_oracle.so"
# strict IEEE: no contraction into fused multiply-adds, no fast-math
CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC"]

_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        LIB.parent.mkdir(exist_ok=True)
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(["gcc", *CFLAGS, "-o", str(tmp), str(SRC), "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        lib.farq_oracle_rows.restype = None
        lib.farq_oracle_rows.argtypes = [ctypes.c_void_p] * 7 + [
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_float, ctypes.c_int]
        _lib = lib
    return _lib


def fused_add_rmsnorm_group_quant_c(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                                    eps: float, group_size: int, q_mode: str = "int8",
                                    ue8m0: bool = False, write_norm: bool = True,
                                    threads: int = 0):
    """Same results as oracle.farq_oracle.fused_add_rmsnorm_group_quant_ref
    (residual_out in x's dtype, norm_out bf16 or None, q int8 / e4m3 bytes,
    scale fp32), computed in C with `threads` OpenMP threads (0 = all)."""
    assert x.dtype in (torch.bfloat16, torch.float16) and residual.dtype == x.dtype
    x = x.detach().cpu().contiguous()
    residual = residual.detach().cpu().contiguous()
    g = gamma.detach().cpu().float().contiguous()
    M, D = x.shape
    G = int(group_size)
    assert D % G == 0 and D <= 16384
    ro = torch.empty_like(x)
    no = torch.empty(M, D, dtype=torch.bfloat16) if write_norm else None
    q = torch.empty(M, D, dtype=torch.uint8)
    s = torch.empty(M, D // G, dtype=torch.float32)
    if threads <= 0:
        threads = len(os.sched_getaffinity(0))
    _load().farq_oracle_rows(
        x.data_ptr(), residual.data_ptr(), g.data_ptr(), ro.data_ptr(),
        no.data_ptr() if no is not None else None, q.data_ptr(), s.data_ptr(),
        M, D, G, 0 if x.dtype == torch.bfloat16 else 1, 1 if q_mode == "e4m3" else 0,
        1 if ue8m0 else 0, float(eps), int(threads))
    if q_mode == "int8":
        q = q.view(torch.int8)
    return ro, no, q, s
