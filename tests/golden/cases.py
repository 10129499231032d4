"""Golden cases: shapes and seeded inputs shared by make_golden.py (which
runs the reference kernels once, in this repository's build container) and
the tests (which regenerate the same inputs and compare against the stored
outputs). Each case names the reference kernel its shape routes to on an
NVIDIA device (src/task01_fused_add_rmsnorm_group_quant.py:1772-1817, :1656-1727).
"""
from __future__ import annotations

import hashlib

import torch

from flagos_kernelgen_72h_shanghai_2026_b200.workloads import Workload, make_inputs

# name -> (workload, rows forced to zero in x and residual, reference kernel)
CASES = {
    "full_row_128x4096_g128_bf16": (
        Workload("g1", 128, 4096, q_dtype=torch.int8, seed=0), (), "_preweighted_full_row_kernel"),
    "segmented_128x7168_g128_bf16": (
        Workload("g2", 128, 7168, q_dtype=torch.int8, res_std=2.0, seed=1), (),
        "_preweighted_segmented_streaming_kernel"),
    "rowgroup_512x5120_g64_fp16": (
        Workload("g3", 512, 5120, dtype=torch.float16, group_size=64, eps=1e-5,
                 gamma_std=0.05, q_dtype=torch.int8, seed=2), (),
        "_nvidia_parallel_row_group_streaming_kernel"),
    "full_row_5x8192_g256_zero_row": (
        Workload("g4", 5, 8192, group_size=256, q_dtype=torch.int8, seed=3), (2,),
        "_preweighted_full_row_kernel"),
    "segmented_160x7168_outliers": (
        Workload("g5", 160, 7168, q_dtype=torch.int8, res_std=2.0, outlier_channels=8,
                 outlier_row_frac=0.01, seed=4), (),
        "_preweighted_segmented_streaming_kernel"),
    "rowgroup_513x4096_g256_fp16_oddM": (
        Workload("g6", 513, 4096, dtype=torch.float16, group_size=256, q_dtype=torch.int8,
                 seed=5), (),
        "_nvidia_parallel_row_group_streaming_kernel"),
    "segmented_130x8192_g256_4seg": (
        Workload("g8", 130, 8192, group_size=256, q_dtype=torch.int8, res_std=2.0, seed=7), (),
        "_preweighted_segmented_streaming_kernel"),
    "rowgroup_512x6144_g128_3seg": (
        Workload("g9", 512, 6144, q_dtype=torch.int8, seed=8), (),
        "_nvidia_parallel_row_group_streaming_kernel"),
    "full_row_1x4096_g128": (
        Workload("g7", 1, 4096, q_dtype=torch.int8, seed=6), (), "_preweighted_full_row_kernel"),
    # the DeepSeek-V3 benchmark shape (4096 x 7168, residual std 2) in int8
    "segmented_4096x7168_dsv3_rows": (
        Workload("g10", 4096, 7168, q_dtype=torch.int8, res_std=2.0, seed=9), (),
        "_preweighted_segmented_streaming_kernel"),
}

# Cases whose fixture keeps every n-th row of q and x_scale only (the whole
# call is run; the stored rows keep the fixture small).
ROW_STEP = {"segmented_4096x7168_dsv3_rows": 32}


def stored_rows(name: str, t: torch.Tensor) -> torch.Tensor:
    """The rows of a full [M, ...] output that the case's fixture stores."""
    return t[::ROW_STEP.get(name, 1)]


def case_inputs(name: str):
    """(workload, x, residual, gamma) on CPU for a golden case."""
    w, zero_rows, _ = CASES[name]
    x, r, g = make_inputs(w)
    for z in zero_rows:
        x[z] = 0
        r[z] = 0
    return w, x, r, g


def input_digest(x: torch.Tensor, r: torch.Tensor, g: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in (x, r, g):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()
