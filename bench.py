"""Benchmark: fused residual-add + RMSNorm + per-token group quantisation on B200.

Metric: achieved HBM GB/s (algorithmic bytes / device time) and us/call at
T x 7168, on 1/2/4/8 GPUs (one process per GPU, rows sharded, no collective
inside the timed region). One step = one call of the operator over one
batch of synthetic input already resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

Under torchrun (N > 1) every rank runs its own shard of rows; rank 0 prints
one JSON line. ``--impl reference`` times the CPU restatement of the
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


def profiled_traffic(workload: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of this workload, if any."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        text = f.read_text()
        if f"workload: {workload}" not in text:
            continue
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", text)
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/farq_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
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
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": w.name, "M": w.M, "D": w.D, "group_size": w.group_size,
                   "q_dtype": str(w.q_dtype).replace("torch.", ""), "rows_per_step": rows},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
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
    per_set = bytes_per_call(rows, w.D, w.group_size)
    nsets = max(2, -(-(3 * L2_BYTES) // per_set)) if per_set < 3 * L2_BYTES else 1
    nsets = min(nsets, 64)
    x0, r0, g = make_inputs(w, device=dev, row_start=start, row_stop=stop, seed_offset=rank)
    sets = []
    for i in range(nsets):
        x = x0 if i == 0 else x0.roll(i, dims=0).contiguous()
        r = r0 if i == 0 else r0.roll(i, dims=0).contiguous()
        sets.append((x, r) + alloc_outputs(w, rows, dev))
    eps, G = w.eps, w.group_size

    def step(i):
        x, r, ro, no, q, s = sets[i % nsets]
        fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, eps, G, ue8m0=w.ue8m0)

    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)

    K = args.steps
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(smi_index(local)) as clocks:
        t_begin.record(stream)
        for i in range(K):
            step(i)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    total_ms = t_begin.elapsed_time(t_end)
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

    # ---- end to end: pinned host inputs -> device -> operator -> host outputs
    e2e = run_e2e(args, w, rows, dev, g, start, rank, pg)

    times = torch.tensor([total_ms, kern_ms, iso_ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
        e2e_t = torch.tensor([e2e["ms"]], dtype=torch.float64, device=dev)
        pg.all_reduce(e2e_t, op=pg.ReduceOp.MAX)
        e2e["ms"] = float(e2e_t.item())
        clk_all = [None] * world
        pg.all_gather_object(clk_all, clk)
    else:
        clk_all = [clk]
    total_ms, kern_ms, iso_ms = float(times[0]), float(times[1]), float(times[2])
    ms_per_step = total_ms / K
    total_rows = rows * world if args.scaling == "weak" else w.M
    job_bytes = bytes_per_call(total_rows, w.D, w.group_size) + (world - 1) * 2 * w.D
    value = job_bytes / (ms_per_step * 1e-3) / 1e9
    kernel_bytes = per_set
    achieved = kernel_bytes / (kern_ms * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    e2e_gbs = job_bytes / (e2e["ms"] * 1e-3) / 1e9

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
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "us_per_call": kern_ms * 1e3, "us_per_call_isolated": iso_ms * 1e3,
        "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "fp16",
        "data": "synthetic (seeded torch.randn on device)",
        "config": {"workload": w.name, "M_per_gpu": rows, "D": w.D, "group_size": w.group_size,
                   "q_dtype": str(w.q_dtype).replace("torch.", ""), "ue8m0": w.ue8m0,
                   "norm_out": False, "bytes_per_call": kernel_bytes,
                   "l2": f"rotating {nsets} input/output sets "
                         f"({nsets * per_set / 1e6:.0f} MB > {L2_BYTES / 1e6:.0f} MB L2)",
                   "parallelism": f"rows sharded over {world} GPU(s), no collective"},
        "pct_of_8tbs_nominal": round(100 * value / world / 8000.0, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": profiled_traffic(w.name)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_gbs, 3), "unit": "GB/s", "ms_per_step": e2e["ms"],
                "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"]},
        "gpu_launches": K,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                   "sm_max_mhz": clk_all[0]["sm_max_mhz"],
                   "reasons": sorted({r for c in clk_all for r in c["reasons"]}),
                   "samples": sum(c["samples"] for c in clk_all)},
    }
    print(json.dumps(line), flush=True)


def run_e2e(args, w, rows, dev, g, start, rank, pg):
    """Same metric through the public host-buffer API: every step copies x and
    residual from pinned host memory to the GPU, runs the operator and copies
    residual_out, x_q and x_scale back to pinned host memory, all inside the
    timed region (the API pipelines row chunks so both PCIe directions and the
    kernel overlap)."""
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant_host

    x, r, _ = make_inputs(w, device=dev, row_start=start, row_stop=start + rows, seed_offset=rank)
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    hr = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
    hx.copy_(x)
    hr.copy_(r)
    del x, r
    hro = torch.empty(hx.shape, dtype=hx.dtype, pin_memory=True)
    hq = torch.empty(hx.shape, dtype=w.q_dtype, pin_memory=True)
    hs = torch.empty(rows, w.groups, dtype=torch.float32, pin_memory=True)
    stream = torch.cuda.current_stream(dev)

    def step():
        fused_add_rmsnorm_group_quant_host(hx, hr, g, hro, None, hq, hs, w.eps, w.group_size,
                                           ue8m0=w.ue8m0, device=dev,
                                           chunk_rows=args.e2e_chunk_rows)

    for _ in range(3):
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
    h2d = hx.numel() * hx.element_size() + hr.numel() * hr.element_size()
    d2h = sum(t.numel() * t.element_size() for t in (hro, hq, hs))
    return {"ms": t0.elapsed_time(t1) / n, "h2d": h2d, "d2h": d2h}


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

    res = {}
    for name, f in (("fused", fused), ("nccl_allreduce_then_kernel", unfused)):
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


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="rows", choices=["rows", "tp"],
                    help="rows: the operator on row shards (default benchmark); tp: the "
                         "tensor-parallel variant (all-reduce fused with the operator)")
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="weak: every GPU runs the full config (default except config 5); "
                         "strong: the config's rows are split over the GPUs (default for config 5)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--e2e-chunk-rows", type=int, default=512)
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the CPU baseline sample")
    ap.add_argument("--ref-budget", type=float, default=90.0,
                    help="seconds of CPU work for the whole --impl reference run")
    ap.add_argument("--no-cpu", action="store_true")
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
    if args.mode == "tp":
        run_tp(args, w, rank, world, local)
        return
    if args.impl == "reference":
        run_reference_arm(args, w, rank, world)
    else:
        run_ours(args, w, rank, world, local)


if __name__ == "__main__":
    main()
