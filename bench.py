"""Benchmark: fused residual-add + RMSNorm + per-token group quantisation on B200.

Metric: achieved HBM GB/s (algorithmic bytes / device time) and us/call at
T x 7168, on 1/2/4/8 GPUs (one process per GPU, rows sharded, no collective
inside the timed region). One step = one call of the operator over one
batch of synthetic input already resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 5] [--impl ours|reference]

Default workload: config 5, 262144 x 7168 bf16 rows split evenly over the N
GPUs (strong scaling, no collective in the timed region); the DeepSeek-V3
4096 x 7168 call on one GPU (config 2) is timed as well and reported beside
it. Under torchrun (N > 1) every rank runs its own slab of rows; rank 0
prints one JSON line. ``--impl reference`` times the CPU restatement of the
reference's math (the reference itself is Triton-only and ships no CPU code;
oracle/farq_oracle.c, OpenMP) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from flagos_kernelgen_72h_shanghai_2026_b200.sharding import shard_rows  # noqa: E402
from flagos_kernelgen_72h_shanghai_2026_b200.workloads import (  # noqa: E402
    CONFIGS, alloc_outputs, bytes_per_call, make_inputs)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
METRIC = "achieved HBM GB/s (% of B200 peak) and us/call at T x 7168, 1/2/4/8 GPUs"
SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def smi_index(local: int) -> str:
    """nvidia-smi -i argument for this process's GPU (honours CUDA_VISIBLE_DEVICES)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


def load_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic_per_row(D: int) -> float | None:
    """DRAM read + write bytes per row of one launch of the row kernel at
    hidden size D, from the committed ncu summary of that kernel (the
    ``traffic_bytes_per_row`` line of a ``profiles/farq_rows_kernel_*`` file
    whose ``hidden: D`` matches). The benchmark's full launches are too large
    to capture under ncu; DRAM traffic of this kernel grows in proportion to
    the rows it processes, so the bench scales this figure by its rows."""
    for f in sorted((ROOT / "profiles").glob("farq_rows_kernel_*.md")):
        text = f.read_text()
        if not re.search(rf"^hidden: {D}$", text, flags=re.M):
            continue
        m = re.search(r"traffic_bytes_per_row:\s*([0-9.eE+]+)", text)
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the GPU is under load.

    Started before the warm-up, so that nvidia-smi is already sampling when
    the timed region begins (no idle gap is inserted for it)."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/farq_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.idx)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        sm, smax, reasons = [], None, set()
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(REASON_NAMES, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def line_config(w, world: int, scaling: str) -> dict:
    """`config` of the JSON line; identical for the repo arm and the reference
    arm at the same workload and N, so the driver can pair them."""
    start, stop = shard_rows(w.M, world, 0) if scaling == "strong" else (0, w.M)
    return {"workload": w.name, "M": w.M if scaling == "strong" else w.M * world,
            "M_per_gpu": stop - start, "D": w.D, "group_size": w.group_size,
            "io_dtype": "bf16" if w.dtype == torch.bfloat16 else "fp16",
            "q_dtype": str(w.q_dtype).replace("torch.", ""), "ue8m0": w.ue8m0,
            "norm_out": False,
            "bytes_per_call": job_bytes(w, world, scaling),
            "parallelism": f"rows sharded over {world} GPU(s), no collective"}


def job_bytes(w, world: int, scaling: str) -> int:
    """Algorithmic bytes of one step of the whole job: every row once, plus
    one gamma read per GPU."""
    total_rows = w.M if scaling == "strong" else w.M * world
    return bytes_per_call(total_rows, w.D, w.group_size) + (world - 1) * 2 * w.D


# Both arms compute in fp32 (fp64 sum of squares on the GPU) on 2-byte inputs.
LINE_DTYPE = "fp32"


# ------------------------------------------------------------------ CPU arm
def cpu_sample(w, steps: int, warmup: int, budget_s: float, min_rows: int = 1):
    """Time the plain-C restatement of the reference math (oracle/farq_oracle.c,
    OpenMP over rows, all host threads) on a bounded row sample of ``w``:
    rows per step sized so that steps + warmup calls take about ``budget_s``
    seconds, but never fewer than ``min_rows`` (small samples would measure
    per-call overhead rather than throughput).
    Returns (GB/s, seconds per step, rows, cores)."""
    from oracle.c_oracle import fused_add_rmsnorm_group_quant_c
    cores = len(os.sched_getaffinity(0))
    mode = "e4m3" if w.q_dtype == torch.float8_e4m3fn else "int8"

    def call(x, r, g):
        fused_add_rmsnorm_group_quant_c(x, r, g, w.eps, w.group_size, mode, w.ue8m0,
                                        write_norm=False, threads=cores)

    probe_rows = min(256, w.M)
    x, r, g = make_inputs(w.with_rows(probe_rows))
    call(x, r, g)
    t0 = time.perf_counter()
    call(x, r, g)
    per_row = (time.perf_counter() - t0) / probe_rows
    rows = int(budget_s / max(1, steps + warmup) / max(per_row, 1e-9))
    rows = max(min_rows, min(w.M, rows))
    x, r, g = make_inputs(w.with_rows(rows))
    for _ in range(warmup):
        call(x, r, g)
    t0 = time.perf_counter()
    for _ in range(steps):
        call(x, r, g)
    dt = (time.perf_counter() - t0) / steps
    b = bytes_per_call(rows, w.D, w.group_size)
    return b / dt / 1e9, dt, rows, cores


def run_reference_arm(args, w, rank, world):
    if rank != 0:
        return
    gbs, dt, rows, cores = cpu_sample(w, args.steps, args.warmup, budget_s=args.ref_budget,
                                      min_rows=16)
    sample = (f"{rows} of {w.M} rows of {w.name} per step, plain-C port of the reference math "
              f"(oracle/farq_oracle.c, OpenMP, {cores} threads)")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "ms_per_full_call_extrapolated": dt * 1e3 * (w.M / rows),
        "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": LINE_DTYPE, "data": "synthetic",
        "config": line_config(w, world, args.scaling),
        "rows_per_step": rows,
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def rotating_sets(w, rows, start, rank, dev):
    """Input/output sets for ``rows`` rows, enough of them that consecutive
    steps never find their inputs in the 126 MB L2 (one set suffices when a
    set is itself several times larger than L2)."""
    per_set = bytes_per_call(rows, w.D, w.group_size)
    nsets = 1 if per_set >= 3 * L2_BYTES else min(64, max(2, -(-(3 * L2_BYTES) // per_set)))
    x0, r0, g = make_inputs(w, device=dev, row_start=start, row_stop=start + rows,
                            seed_offset=rank)
    sets = []
    for i in range(nsets):
        x = x0 if i == 0 else x0.roll(i, dims=0).contiguous()
        r = r0 if i == 0 else r0.roll(i, dims=0).contiguous()
        sets.append((x, r) + alloc_outputs(w, rows, dev))
    return sets, g, per_set


def timed_steps(step, K, W, stream, dev, pg, min_warm_s):
    """W warm-up steps (extended until the GPU has been busy for at least
    ``min_warm_s``, so clocks and memory are at their loaded state), then
    exactly K steps between two CUDA events, with a barrier and a device
    synchronize on both sides. Returns (total ms, warm-up steps run)."""
    w0 = torch.cuda.Event(enable_timing=True)
    w1 = torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for i in range(W):
        step(i)
    w1.record(stream)
    torch.cuda.synchronize(dev)
    warm_ms = w0.elapsed_time(w1)
    extra = 0
    if warm_ms < min_warm_s * 1e3:
        extra = int((min_warm_s * 1e3 - warm_ms) / max(warm_ms / W, 1e-3)) + 1
        for i in range(extra):
            step(W + i)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    return t0.elapsed_time(t1), W + extra


def run_ours(args, w, rank, world, local):
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant
    from flagos_kernelgen_72h_shanghai_2026_b200._build import build_lib

    build_lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    if args.scaling == "strong":
        start, stop = shard_rows(w.M, world, rank)
    else:
        start, stop = 0, w.M
    rows = stop - start
    sets, g, per_set = rotating_sets(w, rows, start, rank, dev)
    nsets = len(sets)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        x, r, ro, no, q, s = sets[i % nsets]
        fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, w.eps, w.group_size, ue8m0=w.ue8m0)

    K = args.steps
    with ClockSampler(smi_index(local)) as clocks:
        total_ms, warm_run = timed_steps(step, K, args.warmup, stream, dev, pg, args.min_warm_s)
    # Each step is exactly one launch of the operator's kernel, so the
    # kernel's average duration over the timed region is total / K.
    kern_ms = total_ms / K
    clk = clocks.summary()
    # Isolated launches (an event pair around each, which serialises the
    # launches), reported beside the back-to-back figure.
    n_iso = min(200, K)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_iso)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_iso)]
    for i in range(n_iso):
        starts[i].record(stream)
        step(i)
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    iso_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / n_iso
    del sets, step

    # ---- the DeepSeek-V3 shape (config 2, 4096 x 7168) on every GPU, per GPU
    dsv3 = None
    if not args.no_dsv3 and w.name != CONFIGS[2].name:
        w2 = CONFIGS[2]
        sets2, g2, per2 = rotating_sets(w2, w2.M, 0, rank, dev)

        def step2(i):
            x, r, ro, no, q, s = sets2[i % len(sets2)]
            fused_add_rmsnorm_group_quant(x, r, g2, ro, no, q, s, w2.eps, w2.group_size)

        k2 = max(K, 200)
        ms2, warm2 = timed_steps(step2, k2, args.warmup, stream, dev, pg, args.min_warm_s)
        dsv3 = {"workload": w2.name, "M_per_gpu": w2.M, "steps": k2, "warmup": warm2,
                "us_per_call": ms2 / k2 * 1e3, "bytes_per_call": per2}
        del sets2, step2

    # ---- the next scope row: the DSA top-k page-table transform at its
    # largest competition shape, on every GPU (per GPU, device time)
    topk = None if args.no_topk else topk_side_leg(args, rank, dev, stream, pg)

    # ---- end to end: pinned host inputs -> device -> operator -> host outputs
    e2e = run_e2e(args, w, rows, dev, g, start, rank, pg)

    # ---- N > 1: the tensor-parallel variant (all-reduce fused with the
    # operator) at the DeepSeek-V3 shape, checked and timed on every rank
    tp = tp_leg(rank, world, dev, pg) if (world > 1 and not args.no_tp) else None

    times = torch.tensor([total_ms, kern_ms, iso_ms, e2e["ms"],
                          dsv3["us_per_call"] if dsv3 else 0.0,
                          topk["us_per_call"] if topk else 0.0], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
        clk_all = [None] * world
        pg.all_gather_object(clk_all, clk)
    else:
        clk_all = [clk]
    total_ms, kern_ms, iso_ms, e2e_ms = (float(times[i]) for i in range(4))
    ms_per_step = total_ms / K
    jb = job_bytes(w, world, args.scaling)
    value = jb / (ms_per_step * 1e-3) / 1e9
    # per-launch figures of the slowest rank: its slab is the largest one
    if args.scaling == "strong":
        a, b = shard_rows(w.M, world, world - 1)
        launch_rows = b - a
    else:
        launch_rows = rows
    kernel_bytes = bytes_per_call(launch_rows, w.D, w.group_size)
    achieved = kernel_bytes / (kern_ms * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    e2e_gbs = jb / (e2e_ms * 1e-3) / 1e9
    if topk:
        topk["us_per_call"] = round(float(times[5]), 2)  # max over ranks
        topk["gbs_per_gpu"] = round(topk["bytes_per_call"] / (float(times[5]) * 1e-6) / 1e9, 2)
        topk["frac_of_peak"] = round(topk["gbs_per_gpu"] / load_peak()[0], 4)
    if dsv3:
        dsv3["us_per_call"] = float(times[4])  # max over ranks
        dsv3["gbs_per_gpu"] = round(dsv3["bytes_per_call"] / (dsv3["us_per_call"] * 1e-6) / 1e9, 2)
        dsv3["frac_of_peak"] = round(dsv3["gbs_per_gpu"] / peak, 4)
        dsv3["peak_kind"] = peak_kind

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, dt, srows, cores = cpu_sample(w, 3, 1, budget_s=args.cpu_budget)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"{srows} rows of {w.name} per call, plain-C port of the reference math "
                         f"(oracle/farq_oracle.c, OpenMP, {cores} threads), 3 timed calls"}
    if pg:
        pg.destroy_process_group()
    if rank != 0:
        return
    sm = [c["sm_mhz"] for c in clk_all if c["sm_mhz"]]
    cfg = line_config(w, world, args.scaling)
    traffic_row = profiled_traffic_per_row(w.D)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": K, "warmup": warm_run, "ms_per_step": ms_per_step,
        "us_per_call": kern_ms * 1e3, "us_per_call_isolated": iso_ms * 1e3,
        "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": LINE_DTYPE,
        "data": "synthetic (seeded torch.randn on device)",
        "config": cfg,
        "l2": (f"inputs larger than L2: {nsets} rotating input/output set(s) of "
               f"{per_set / 1e6:.0f} MB per GPU (L2 {L2_BYTES / 1e6:.0f} MB)"),
        "pct_of_8tbs_nominal": round(100 * value / world / 8000.0, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": round(traffic_row * launch_rows) if traffic_row else None,
                     "traffic_source": "ncu per-row DRAM bytes of a smaller capture x rows per "
                                       "launch" if traffic_row else None},
        "dsv3_4096x7168_per_gpu": dsv3,
        "tp_allreduce_fused_4096x7168": tp,
        "dsa_topk_per_gpu": topk,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_gbs, 3), "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": e2e["h2d"] * world, "d2h_bytes_per_step": e2e["d2h"] * world,
                "host_staging_rows_per_gpu": e2e["stage_rows"]},
        "gpu_launches": K,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                   "sm_max_mhz": clk_all[0]["sm_max_mhz"],
                   "reasons": sorted({r for c in clk_all for r in c["reasons"]}),
                   "samples": sum(c["samples"] for c in clk_all),
                   "window": "warm-up and timed region (sampler started before the warm-up)"},
    }
    print(json.dumps(line), flush=True)


def topk_side_leg(args, rank, dev, stream, pg) -> dict:
    """Task 02 (dsa_topk_page_table_transform) at its largest competition
    shape (fp32 scores, 32768 rows x 4096 blocks, K = 128) on this GPU:
    back-to-back launches between CUDA events after a warm-up, rotating
    score sets over 3x L2. Reported beside the main line; `--mode topk` is
    the full measurement of that path."""
    from flagos_kernelgen_72h_shanghai_2026_b200 import dsa_topk_page_table_transform
    from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import (
        TOPK_CONFIGS, make_topk_inputs, topk_bytes_per_call)

    w = TOPK_CONFIGS["t2_nb4096_k128_2x32x512"]
    per = topk_bytes_per_call(w)
    nsets = 1 if per >= 3 * L2_BYTES else min(16, max(2, -(-(3 * L2_BYTES) // per)))
    s, pt, qp, kv = make_topk_inputs(w.with_(seed=w.seed + rank), device=dev)
    sets = [(s if i == 0 else s.roll(i, dims=2).contiguous()) for i in range(nsets)]
    ob = torch.empty(w.B, w.H, w.Q, w.top_k, dtype=torch.int32, device=dev)
    op = torch.empty_like(ob)

    def step(i):
        dsa_topk_page_table_transform(sets[i % nsets], pt, qp, kv, ob, op, w.block_size, w.top_k)

    k = 200
    ms, warm = timed_steps(step, k, args.warmup, stream, dev, pg, args.min_warm_s)
    return {"workload": w.name, "steps": k, "warmup": warm, "us_per_call": ms / k * 1e3,
            "bytes_per_call": per, "dtype": "fp32 scores, int32 ids and pages"}


def tp_leg(rank, world, dev, pg, steps: int = 100, warmup: int = 20) -> dict:
    """Tensor-parallel variant (tp.TPFusedNormQuant, farq_ar_launch) on all N
    ranks at 4096 x 7168: x = bf16(sum of the N ranks' partials) fused with
    the operator, every output row replicated to every rank. Checked on every
    rank against the single-GPU kernel applied to the same x (computed
    locally from the seeded partials: residual_out bit-exact, scales within
    1e-6 relative, q within one e4m3 step on at most 0.1 % of elements), then
    timed against NCCL all-reduce + the single-GPU kernel (device time, max
    over ranks). Runs after the main timing; not part of `value`."""
    import torch.distributed as dist
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant
    from flagos_kernelgen_72h_shanghai_2026_b200.tp import TPFusedNormQuant

    w = CONFIGS[2]
    M, D, G = w.M, w.D, w.group_size
    op = TPFusedNormQuant(M, D, G, dtype=w.dtype, q_dtype=w.q_dtype)

    def partial(k):
        gen = torch.Generator().manual_seed(7000 + k)
        return torch.randn(M, D, generator=gen).to(w.dtype)

    gen = torch.Generator().manual_seed(6999)
    residual = (2 * torch.randn(M, D, generator=gen)).to(w.dtype).to(dev)
    gamma = (1 + 0.1 * torch.randn(D, generator=gen)).to(w.dtype).to(dev)
    mine = partial(rank).to(dev)
    op.partial_buffer(M).copy_(mine)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ro, _, q, s = op(M, residual, gamma, w.eps, status=status)
    torch.cuda.synchronize(dev)
    # reference on this GPU: x in rank order, summed in fp32, rounded once
    x = torch.zeros(M, D, dtype=torch.float32, device=dev)
    for k in range(world):
        x += (mine if k == rank else partial(k).to(dev)).float()
    x = x.to(w.dtype)
    rro, rno, rq, rs = alloc_outputs(w, M, dev)
    fused_add_rmsnorm_group_quant(x, residual, gamma, rro, rno, rq, rs, w.eps, G)
    torch.cuda.synchronize(dev)
    ok = int(status.item()) == 0 and torch.equal(ro.view(torch.int16), rro.view(torch.int16))
    ok = ok and float(((s - rs).abs() / rs.abs()).max()) <= 1e-6

    def ordered(b):
        b = b.view(torch.uint8).to(torch.int32)
        return torch.where(b >= 128, -(b & 127), b)

    dq = (ordered(q) - ordered(rq)).abs()
    ok = ok and int(dq.max()) <= 1 and float((dq != 0).float().mean()) <= 1e-3
    del x, rno
    xr = torch.empty_like(mine)

    def fused():
        op(M, residual, gamma, w.eps)

    def unfused():
        xr.copy_(mine)
        dist.all_reduce(xr)
        fused_add_rmsnorm_group_quant(xr, residual, gamma, rro, None, rq, rs, w.eps, G)

    res = []
    for f in (fused, unfused):
        for _ in range(warmup):
            f()
        torch.cuda.synchronize(dev)
        pg.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            f()
        t1.record()
        torch.cuda.synchronize(dev)
        res.append(t0.elapsed_time(t1) / steps * 1e3)
    out = torch.tensor(res + [0.0 if ok else 1.0], dtype=torch.float64, device=dev)
    pg.all_reduce(out, op=pg.ReduceOp.MAX)
    return {"world": world, "M": M, "D": D, "fused_us_per_call": round(float(out[0]), 2),
            "nccl_allreduce_then_kernel_us_per_call": round(float(out[1]), 2),
            "check_vs_single_gpu_kernel": "ok" if float(out[2]) == 0.0 else "FAILED",
            "timing": f"{steps} calls between CUDA events after {warmup} warm-ups, max over ranks"}


def run_e2e(args, w, rows, dev, g, start, rank, pg):
    """Same metric through the public host-buffer API: every step copies the
    rank's x and residual rows from pinned host memory to the GPU, runs the
    operator and copies residual_out, x_q and x_scale back to pinned host
    memory, all inside the timed region (the API pipelines row chunks so both
    PCIe directions and the kernel overlap). The pinned buffers hold at most
    ``--e2e-stage-rows`` rows: a larger slab is streamed through them in
    consecutive API calls, so a step still moves every row of the slab."""
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant_host

    stage = min(rows, args.e2e_stage_rows)
    x, r, _ = make_inputs(w, device=dev, row_start=start, row_stop=start + stage,
                          seed_offset=rank)
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    hr = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
    hx.copy_(x)
    hr.copy_(r)
    del x, r
    hro = torch.empty(hx.shape, dtype=hx.dtype, pin_memory=True)
    hq = torch.empty(hx.shape, dtype=w.q_dtype, pin_memory=True)
    hs = torch.empty(stage, w.groups, dtype=torch.float32, pin_memory=True)
    stream = torch.cuda.current_stream(dev)
    pieces = []
    for a in range(0, rows, stage):
        n = min(stage, rows - a)
        pieces.append(n)

    def step():
        for n in pieces:
            fused_add_rmsnorm_group_quant_host(hx[:n], hr[:n], g, hro[:n], None, hq[:n], hs[:n],
                                               w.eps, w.group_size, ue8m0=w.ue8m0, device=dev,
                                               chunk_rows=args.e2e_chunk_rows)

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    n = max(3, min(args.e2e_steps, args.steps))
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    t0.record(stream)
    for _ in range(n):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    per_row_in = w.D * hx.element_size() * 2
    per_row_out = w.D * (hro.element_size() + hq.element_size()) + w.groups * 4
    return {"ms": t0.elapsed_time(t1) / n, "h2d": rows * per_row_in, "d2h": rows * per_row_out,
            "stage_rows": stage}


def run_tp(args, w, rank, world, local):
    """Tensor-parallel variant: x = all-reduce of per-rank partials fused with
    the operator (tp.TPFusedNormQuant), against NCCL all-reduce followed by the
    single-GPU kernel, on the same M x D per call. Prints its own JSON line
    (device time, max over ranks); not the default benchmark."""
    import torch.distributed as dist
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant
    from flagos_kernelgen_72h_shanghai_2026_b200._build import build_lib
    from flagos_kernelgen_72h_shanghai_2026_b200.tp import TPFusedNormQuant

    build_lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29561")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    M, D, G = w.M, w.D, w.group_size
    op = TPFusedNormQuant(M, D, G, dtype=w.dtype, q_dtype=w.q_dtype)
    x, r, g = make_inputs(w, device=dev, seed_offset=rank)
    op.partial_buffer(M).copy_(x)
    xr = torch.empty_like(x)
    ro, no, q, s = alloc_outputs(w, M, dev)

    def fused():
        op(M, r, g, w.eps, ue8m0=w.ue8m0)

    def unfused():
        xr.copy_(x)
        dist.all_reduce(xr)
        fused_add_rmsnorm_group_quant(xr, r, g, ro, no, q, s, w.eps, G, ue8m0=w.ue8m0)

    def fused_kernel_w1():
        op(M, r, g, w.eps, ue8m0=w.ue8m0, _fused_at_world1=True)

    arms = [("fused", fused), ("nccl_allreduce_then_kernel", unfused)]
    if world == 1:  # the default routes world 1 to the single-GPU kernel
        arms.append(("fused_allreduce_kernel_forced_at_world1", fused_kernel_w1))
    res = {}
    for name, f in arms:
        for _ in range(args.warmup):
            f()
        torch.cuda.synchronize(dev)
        dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            f()
        t1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([t0.elapsed_time(t1) / args.steps * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(float(t.item()), 2)
    if rank == 0:
        print(json.dumps({"metric": "tensor-parallel all-reduce + add + RMSNorm + group quant, us/call",
                          "mode": "tp", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "config": {"workload": w.name, "M": M, "D": D, "group_size": G},
                          "us_per_call": res, "higher_is_better": False}), flush=True)
    dist.destroy_process_group()


def run_topk(args, rank, world, local):
    """Task 02, the DSA top-k page-table transform, at its largest competition
    shape (fp32 scores, 32768 rows x 4096 blocks, K = 128). Metric: algorithmic
    HBM GB/s (every candidate score read once, ids and pages written, page
    entries gathered: R * (4 NB + 12 K) + 8 R bytes) and us/call. Rows shard
    over GPUs (weak scaling: every GPU runs the full shape, no collective).
    Prints its own JSON line; not the default benchmark."""
    from flagos_kernelgen_72h_shanghai_2026_b200 import dsa_topk_page_table_transform
    from flagos_kernelgen_72h_shanghai_2026_b200._build import build_topk_lib
    from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import (
        TOPK_CONFIGS, make_topk_inputs, topk_bytes_per_call)

    w = TOPK_CONFIGS[args.topk_config]
    if args.rows > 0:
        w = w.with_(B=1, H=1, Q=args.rows)
    if rank != 0 and args.impl == "reference":
        return
    if args.impl == "reference":
        run_topk_reference(args, w, world)
        return
    build_topk_lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    per = topk_bytes_per_call(w)
    nsets = 1 if per >= 3 * L2_BYTES else min(16, max(2, -(-(3 * L2_BYTES) // per)))
    s, pt, qp, kv = make_topk_inputs(w.with_(seed=w.seed + rank), device=dev)
    sets = [(s if i == 0 else s.roll(i, dims=2).contiguous()) for i in range(nsets)]
    ob = torch.empty(w.B, w.H, w.Q, w.top_k, dtype=torch.int32, device=dev)
    op = torch.empty_like(ob)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        dsa_topk_page_table_transform(sets[i % nsets], pt, qp, kv, ob, op, w.block_size, w.top_k)

    K = args.steps
    with ClockSampler(smi_index(local)) as clocks:
        total_ms, warm_run = timed_steps(step, K, args.warmup, stream, dev, pg, args.min_warm_s)
    clk = clocks.summary()

    # end to end: pinned host scores / page table / positions -> device ->
    # kernel -> ids and pages back to pinned host memory, every step
    hs = torch.empty(s.shape, dtype=s.dtype, pin_memory=True)
    hs.copy_(s)
    hpt, hqp, hkv = (t.cpu().pin_memory() for t in (pt, qp, kv))
    hob = torch.empty(ob.shape, dtype=ob.dtype, pin_memory=True)
    hop = torch.empty_like(hob).pin_memory()
    ds = torch.empty_like(s)
    dpt, dqp, dkv = torch.empty_like(pt), torch.empty_like(qp), torch.empty_like(kv)

    def e2e_step():
        ds.copy_(hs, non_blocking=True)
        dpt.copy_(hpt, non_blocking=True)
        dqp.copy_(hqp, non_blocking=True)
        dkv.copy_(hkv, non_blocking=True)
        dsa_topk_page_table_transform(ds, dpt, dqp, dkv, ob, op, w.block_size, w.top_k)
        hob.copy_(ob, non_blocking=True)
        hop.copy_(op, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    n_e2e = max(3, min(args.e2e_steps, K))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / n_e2e
    h2d = sum(t.numel() * t.element_size() for t in (hs, hpt, hqp, hkv))
    d2h = sum(t.numel() * t.element_size() for t in (hob, hop))

    times = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
        clk_all = [None] * world
        pg.all_gather_object(clk_all, clk)
    else:
        clk_all = [clk]
    total_ms, e2e_ms = float(times[0]), float(times[1])
    ms = total_ms / K
    value = per * world / (ms * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    achieved = per / (ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, dt, rows, cores = topk_cpu_sample(w, budget_s=args.cpu_budget)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"{rows} of {w.rows} rows of {w.name} per call, numpy restatement of "
                         f"the reference (oracle/dsa_topk_oracle.py, single thread)"}
    if pg:
        pg.destroy_process_group()
    if rank != 0:
        return
    sm = [c["sm_mhz"] for c in clk_all if c["sm_mhz"]]
    print(json.dumps({
        "metric": TOPK_METRIC, "mode": "topk", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": world, "steps": K, "warmup": warm_run, "ms_per_step": ms,
        "us_per_call": ms * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded torch.randn scores)",
        "config": topk_line_config(w, world),
        "l2": f"inputs larger than L2: {nsets} rotating score set(s) of {per / 1e6:.0f} MB",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": profiled_topk_traffic(w.name),
                     "traffic_source": "DRAM read + write of one ncu-captured launch of this "
                                       "workload (committed profile)"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(per * world / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world},
        "gpu_launches": K,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                   "sm_max_mhz": clk_all[0]["sm_max_mhz"],
                   "reasons": sorted({r for c in clk_all for r in c["reasons"]}),
                   "samples": sum(c["samples"] for c in clk_all)},
    }), flush=True)


TOPK_METRIC = "DSA top-k page-table transform: algorithmic HBM GB/s and us/call"


def profiled_topk_traffic(workload: str) -> int | None:
    """DRAM read + write bytes of one launch of the top-k kernel on
    ``workload``, from the committed ncu summary of that workload (the
    ``traffic_bytes_per_launch`` line of a ``profiles/dsa_topk_kernel_*``
    file whose ``workload:`` line names it)."""
    for f in sorted((ROOT / "profiles").glob("dsa_topk_kernel_*.md")):
        text = f.read_text()
        if not re.search(rf"^workload: {re.escape(workload)}\b", text, flags=re.M):
            continue
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", text)
        if m:
            return int(m.group(1))
    return None


def topk_line_config(w, world):
    from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import topk_bytes_per_call
    return {"workload": w.name, "B": w.B, "H": w.H, "Q": w.Q, "NB": w.NB, "top_k": w.top_k,
            "block_size": w.block_size, "scores_dtype": str(w.dtype).replace("torch.", ""),
            "bytes_per_call": topk_bytes_per_call(w) * world,
            "parallelism": f"full shape on each of {world} GPU(s), no collective"}


def topk_cpu_sample(w, budget_s: float):
    """Time the numpy restatement of the reference (the oracle) on a bounded
    row sample of ``w``. Returns (GB/s, seconds per call, rows, cores)."""
    from oracle.dsa_topk_oracle import dsa_topk_page_table_transform_ref
    from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import (
        make_topk_inputs, topk_bytes_per_call)
    probe = w.with_(B=1, H=1, Q=min(256, w.rows))
    s, pt, qp, kv = make_topk_inputs(probe)
    t0 = time.perf_counter()
    dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    per_row = (time.perf_counter() - t0) / probe.rows
    rows = max(64, min(w.rows, int(budget_s / 4 / max(per_row, 1e-9))))
    sample = w.with_(B=1, H=1, Q=rows)
    s, pt, qp, kv = make_topk_inputs(sample)
    dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    t0 = time.perf_counter()
    for _ in range(3):
        dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    dt = (time.perf_counter() - t0) / 3
    return topk_bytes_per_call(sample) / dt / 1e9, dt, rows, 1


def run_topk_reference(args, w, world):
    """Reference arm of --mode topk: the reference is Triton-only (no CPU code
    of its own), so its CPU stand-in is the numpy restatement, timed on a
    bounded row sample, rank 0 only."""
    gbs, dt, rows, cores = topk_cpu_sample(w, budget_s=args.ref_budget / 3)
    sample = (f"{rows} of {w.rows} rows of {w.name} per step, numpy restatement of the "
              f"reference (oracle/dsa_topk_oracle.py, single thread)")
    print(json.dumps({
        "metric": TOPK_METRIC, "mode": "topk", "value": round(gbs, 3), "unit": "GB/s",
        "impl": "reference", "n_gpus": world, "steps": 3, "warmup": 1,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic", "config": topk_line_config(w, world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_pcie(args, rank, world, local):
    """Host-link ceiling of the end-to-end leg: bare pinned-memory copies of
    the e2e leg's bytes (x and residual in, residual_out, x_q and x_scale
    out, for --e2e-stage-rows rows of the workload), both directions at once
    on two streams, on every rank at the same time. Prints one JSON line:
    aggregate GB/s of the workload's algorithmic bytes moved at that copy
    speed (comparable with the e2e value), and the raw copy GB/s per
    direction. Not the default benchmark."""
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    w = CONFIGS[args.config]
    a, b = shard_rows(w.M, world, rank) if args.scaling == "strong" else (0, w.M)
    rows = min(args.e2e_stage_rows, b - a)
    esz = 2
    h2d = rows * w.D * esz * 2
    d2h = rows * (w.D * esz + w.D + w.groups * 4)
    hin = torch.empty(h2d, dtype=torch.uint8, pin_memory=True)
    hout = torch.empty(d2h, dtype=torch.uint8, pin_memory=True)
    din = torch.empty(h2d, dtype=torch.uint8, device=dev)
    dout = torch.empty(d2h, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    res = {}
    for mode in ("h2d", "d2h", "both"):
        def step():
            if mode in ("h2d", "both"):
                with torch.cuda.stream(s_in):
                    din.copy_(hin, non_blocking=True)
            if mode in ("d2h", "both"):
                with torch.cuda.stream(s_out):
                    hout.copy_(dout, non_blocking=True)
        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
        t0 = time.perf_counter()
        n = max(3, args.steps // 10)
        for _ in range(n):
            step()
        torch.cuda.synchronize(dev)
        dt = torch.tensor([(time.perf_counter() - t0) / n], dtype=torch.float64, device=dev)
        if pg:
            pg.all_reduce(dt, op=pg.ReduceOp.MAX)
        res[mode] = float(dt)
    if pg:
        pg.destroy_process_group()
    if rank != 0:
        return
    alg = bytes_per_call(rows, w.D, w.group_size) * world
    print(json.dumps({
        "metric": "host-link ceiling of the e2e leg: bare pinned copies on every rank at once",
        "mode": "pcie", "n_gpus": world, "rows_per_gpu": rows,
        "h2d_gbs_per_gpu": round(h2d / res["h2d"] / 1e9, 2),
        "d2h_gbs_per_gpu": round(d2h / res["d2h"] / 1e9, 2),
        "both_ms": res["both"] * 1e3,
        "aggregate_copy_gbs_both": round((h2d + d2h) * world / res["both"] / 1e9, 2),
        "ceiling_algorithmic_gbs": round(alg / res["both"] / 1e9, 2),
        "timing": "host clock around K copy rounds after a device sync, max over ranks",
    }), flush=True)


def run_latency(args, local):
    """Small-M latency regime (M <= 128, where the reference's launch
    overhead dominates): host microseconds per eager call (the Python
    wrapper and its C++ launch path; beside it the ctypes path with and
    without its argument-struct cache; host clock over calls issued back to
    back), device microseconds per call (CUDA events,
    eager), and device microseconds per call when the calls are replayed from
    one CUDA graph. Prints its own JSON line; not the default benchmark."""
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant
    from flagos_kernelgen_72h_shanghai_2026_b200._build import build_lib

    build_lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    res = {}
    for M in (1, 32, 128):
        w = CONFIGS[2].with_rows(M)
        x, r, g = make_inputs(w, device=dev)
        ro, no, q, s = alloc_outputs(w, M, dev)

        def call():
            fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, w.eps, w.group_size)

        for _ in range(50):
            call()
        torch.cuda.synchronize(dev)
        n = 2000
        t0 = time.perf_counter()
        for _ in range(n):
            call()
        host_us = (time.perf_counter() - t0) / n * 1e6
        torch.cuda.synchronize(dev)
        # the ctypes path (the C++ launch path switched off): with the
        # argument-struct cache, and with it emptied before every call
        from flagos_kernelgen_72h_shanghai_2026_b200 import task01
        fast, task01._fast = task01._fast, None
        try:
            for _ in range(50):
                call()
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(n):
                call()
            host_us_ctypes = (time.perf_counter() - t0) / n * 1e6
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(n):
                task01._tls.args = {}
                call()
            host_us_nocache = (time.perf_counter() - t0) / n * 1e6
            torch.cuda.synchronize(dev)
        finally:
            task01._fast = fast
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            call()
        e1.record()
        torch.cuda.synchronize(dev)
        eager_us = e0.elapsed_time(e1) / n * 1e3
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            call()
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(graph, stream=side):
                for _ in range(100):
                    call()
        torch.cuda.synchronize(dev)
        graph.replay()
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(20):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        graph_us = e0.elapsed_time(e1) / 2000 * 1e3
        res[f"M{M}"] = {"host_us_per_call": round(host_us, 2),
                        "host_us_per_call_ctypes_cached": round(host_us_ctypes, 2),
                        "host_us_per_call_ctypes_uncached": round(host_us_nocache, 2),
                        "device_us_per_call_eager": round(eager_us, 2),
                        "device_us_per_call_graph": round(graph_us, 2)}
    print(json.dumps({"metric": "small-M latency, us/call (D = 7168, bf16 -> e4m3)",
                      "mode": "latency", "n_gpus": 1, "higher_is_better": False,
                      "config": {"workload": "cfg2 shape with M in {1, 32, 128}", "D": 7168},
                      "us_per_call": res}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=5, choices=sorted(CONFIGS),
                    help="workload (default 5: 262144 x 7168 split over the GPUs; the "
                         "DeepSeek-V3 4096 x 7168 per-GPU figure is reported beside it)")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the workload's total rows (small cases for ncu captures)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="rows", choices=["rows", "tp", "latency", "topk", "pcie"],
                    help="rows: the operator on row shards (default benchmark); tp: the "
                         "tensor-parallel variant (all-reduce fused with the operator); "
                         "latency: small-M host and device cost per call; topk: the DSA "
                         "top-k page-table transform (Task 02); pcie: host-link ceiling of the "
                         "e2e leg")
    ap.add_argument("--topk-config", default="t2_nb4096_k128_2x32x512",
                    help="Task 02 workload of --mode topk (topk_workloads.TOPK_CONFIGS)")
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="weak: every GPU runs the full config (default except config 5); "
                         "strong: the config's rows are split over the GPUs (default for config 5)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--e2e-chunk-rows", type=int, default=512)
    ap.add_argument("--e2e-stage-rows", type=int, default=32768,
                    help="rows of pinned host memory per GPU for the e2e leg")
    ap.add_argument("--min-warm-s", type=float, default=0.5,
                    help="extend the warm-up until the GPU has been busy this long")
    ap.add_argument("--no-dsv3", action="store_true",
                    help="skip the extra DeepSeek-V3 4096 x 7168 per-GPU figure")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the CPU baseline sample")
    ap.add_argument("--ref-budget", type=float, default=90.0,
                    help="seconds of CPU work for the whole --impl reference run")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-topk", action="store_true",
                    help="skip the DSA top-k figure reported beside the main line")
    ap.add_argument("--no-tp", action="store_true",
                    help="N > 1: skip the tensor-parallel leg reported beside the main line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.scaling is None:
        args.scaling = "strong" if args.config == 5 else "weak"
    rank, world, local = dist_env()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            ap.error("run N > 1 under torchrun (one process per GPU)")
    w = CONFIGS[args.config]
    if args.rows > 0:
        w = w.with_rows(args.rows)
    if args.mode == "tp":
        run_tp(args, w, rank, world, local)
        return
    if args.mode == "latency":
        run_latency(args, local)
        return
    if args.mode == "topk":
        run_topk(args, rank, world, local)
        return
    if args.mode == "pcie":
        run_pcie(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference_arm(args, w, rank, world)
    else:
        run_ours(args, w, rank, world, local)


if __name__ == "__main__":
    main()
