"""Seeded synthetic inputs for the five benchmark shapes of this operator.

The reference ships no workloads (its competition harness is not part of the
repository); the five configurations below stand in for it. They follow the
shapes the reference routes on NVIDIA parts (task01…py:1772-1817 and
:1656, M = 1-8192, D = 4096-8192, G = 64/128/256 per its slides) and the
DeepSeek-V3 hidden size 7168.

Inputs are generated with ``torch.Generator`` seeded per configuration, in
the order x, residual, gamma (then the outlier indices), so a given seed
gives identical tensors on every machine with this torch build.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    D: int
    dtype: torch.dtype = torch.bfloat16
    group_size: int = 128
    eps: float = 1e-6
    q_dtype: torch.dtype = torch.float8_e4m3fn
    ue8m0: bool = False
    x_std: float = 1.0
    res_std: float = 1.0
    gamma_std: float = 0.1
    outlier_channels: int = 0      # channels of x scaled by outlier_channel_gain
    outlier_channel_gain: float = 100.0
    outlier_row_frac: float = 0.0  # fraction of rows of x scaled by outlier_row_gain
    outlier_row_gain: float = 20.0
    seed: int = 0

    @property
    def groups(self) -> int:
        return self.D // self.group_size

    def with_rows(self, M: int) -> "Workload":
        return replace(self, M=M)


CONFIGS: dict[int, Workload] = {
    1: Workload("cfg1_cpu_ref_128x4096", 128, 4096),
    2: Workload("cfg2_dsv3_4096x7168", 4096, 7168, res_std=2.0),
    3: Workload("cfg3_outlier_16384x7168", 16384, 7168, res_std=2.0,
                outlier_channels=8, outlier_row_frac=0.01),
    4: Workload("cfg4_fp16_g64_ue8m0_8192x5120", 8192, 5120, dtype=torch.float16,
                group_size=64, eps=1e-5, ue8m0=True, gamma_std=0.05),
    5: Workload("cfg5_sharded_262144x7168", 262144, 7168),
}


def make_inputs(w: Workload, device: str | torch.device = "cpu", row_start: int = 0,
                row_stop: int | None = None, seed_offset: int = 0):
    """(x, residual, gamma) for rows [row_start, row_stop) of workload ``w``.

    On CPU the full [M, D] tensors are drawn and sliced, so any row range is
    bit-identical to the same rows of the full draw. On CUDA (large
    benchmark shapes) only the requested rows are drawn, from a generator
    seeded with ``w.seed + seed_offset``; gamma always comes from ``w.seed``.
    """
    row_stop = w.M if row_stop is None else row_stop
    dev = torch.device(device)
    if dev.type == "cpu":
        g = torch.Generator().manual_seed(w.seed)
        x = torch.randn(w.M, w.D, generator=g) * w.x_std
        r = torch.randn(w.M, w.D, generator=g) * w.res_std
        gamma = 1.0 + w.gamma_std * torch.randn(w.D, generator=g)
        x = _outliers(w, x, g)
        return (x[row_start:row_stop].to(w.dtype).contiguous(),
                r[row_start:row_stop].to(w.dtype).contiguous(), gamma.to(w.dtype))
    gg = torch.Generator().manual_seed(w.seed)
    gamma = (1.0 + w.gamma_std * torch.randn(w.D, generator=gg)).to(w.dtype).to(dev)
    g = torch.Generator(device=dev).manual_seed(w.seed + seed_offset)
    rows = row_stop - row_start
    x = torch.empty(rows, w.D, dtype=w.dtype, device=dev)
    r = torch.empty(rows, w.D, dtype=w.dtype, device=dev)
    chunk = 8192
    for s in range(0, rows, chunk):  # bounded fp32 temporaries
        e = min(rows, s + chunk)
        x[s:e] = (torch.randn(e - s, w.D, generator=g, device=dev) * w.x_std).to(w.dtype)
        r[s:e] = (torch.randn(e - s, w.D, generator=g, device=dev) * w.res_std).to(w.dtype)
    if w.outlier_channels or w.outlier_row_frac:
        xf = _outliers(w, x.float(), torch.Generator(device=dev).manual_seed(w.seed + 7))
        x = xf.to(w.dtype)
    return x, r, gamma


def _outliers(w: Workload, x: torch.Tensor, g: torch.Generator) -> torch.Tensor:
    if w.outlier_channels:
        ch = torch.randperm(w.D, generator=g, device=g.device)[: w.outlier_channels].to(x.device)
        x[:, ch] *= w.outlier_channel_gain
    if w.outlier_row_frac:
        n = max(1, int(round(x.shape[0] * w.outlier_row_frac)))
        rows = torch.randperm(x.shape[0], generator=g, device=g.device)[:n].to(x.device)
        x[rows] *= w.outlier_row_gain
    return x


def alloc_outputs(w: Workload, M: int | None = None, device: str | torch.device = "cuda",
                  write_norm: bool = False, norm_dtype: torch.dtype = torch.bfloat16):
    """(residual_out, norm_out or None, x_q, x_scale) for ``M`` rows of ``w``."""
    M = w.M if M is None else M
    ro = torch.empty(M, w.D, dtype=w.dtype, device=device)
    no = torch.empty(M, w.D, dtype=norm_dtype, device=device) if write_norm else None
    q = torch.empty(M, w.D, dtype=w.q_dtype, device=device)
    s = torch.empty(M, w.groups, dtype=torch.float32, device=device)
    return ro, no, q, s


def bytes_per_call(M: int, D: int, group_size: int, in_bytes: int = 2,
                   write_norm: bool = False, norm_bytes: int = 2, gamma_bytes: int = 2,
                   rout_bytes: int | None = None) -> int:
    """Algorithmic HBM bytes of one call: read x, residual, gamma once; write
    residual_out, q (1 B), scales (4 B per group) and, if asked, norm_out.
    = 7N + 4N/G + 2D for 2-byte inputs without norm_out (N = M*D)."""
    rout_bytes = in_bytes if rout_bytes is None else rout_bytes
    N = M * D
    b = 2 * in_bytes * N + gamma_bytes * D + rout_bytes * N + N + 4 * (N // group_size)
    if write_norm:
        b += norm_bytes * N
    return b
