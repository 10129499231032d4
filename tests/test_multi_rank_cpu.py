"""Host-side logic of the row-sharded multi-GPU path, on gloo ranks on CPU.

The device work per rank is the same kernel as on one GPU; what N > 1 adds is
the row partition, the max-over-ranks timing and the handling of a rank that
fails between steps. Those run here as world_size-2 gloo process groups
(the oracle stands in for the per-rank device call)."""
import os
import socket
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from flagos_kernelgen_72h_shanghai_2026_b200.sharding import gather_rows, max_over_ranks, shard_rows
from flagos_kernelgen_72h_shanghai_2026_b200.workloads import Workload, make_inputs

ROOT = str(Path(__file__).resolve().parent.parent)


@pytest.mark.parametrize("M", [0, 1, 7, 128, 4096, 262144, 262147])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(M, world):
    slabs = [shard_rows(M, world, r) for r in range(world)]
    assert slabs[0][0] == 0 and slabs[-1][1] == M
    for (_, b0), (a1, _) in zip(slabs, slabs[1:]):
        assert b0 == a1
    sizes = [b - a for a, b in slabs]
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == M


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    return dist


def _sharded_worker(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        from oracle.farq_oracle import fused_add_rmsnorm_group_quant_ref
        torch.set_num_threads(1)
        dist = _init(rank, world, port)
        w = Workload("mr", 37, 1024, seed=5)
        a, b = shard_rows(w.M, world, rank)
        x, r, g = make_inputs(w, row_start=a, row_stop=b)
        _, _, qq, s = fused_add_rmsnorm_group_quant_ref(x, r, g, w.eps, w.group_size, "e4m3")
        t = max_over_ranks([float(rank + 1), float(10 - rank)])
        full_q = gather_rows(qq, w.M)
        full_s = gather_rows(s, w.M)
        if rank == 0:
            X, R, Gm = make_inputs(w)
            _, _, rq, rs = fused_add_rmsnorm_group_quant_ref(X, R, Gm, w.eps, w.group_size, "e4m3")
            q.put(("ok", bool(torch.equal(full_q, rq) and torch.equal(full_s, rs)), t))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", traceback.format_exc(), None))


def _run(target, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        return q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()


def test_sharded_rows_reassemble_bit_exact_gloo():
    status, ok, t = _run(_sharded_worker)
    assert status == "ok", ok
    assert ok is True
    assert t == [2.0, 10.0]  # element-wise max over ranks


def _failing_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port, timeout_s=20)
        if rank == 1:
            # this rank fails between steps: it leaves without joining the barrier
            os._exit(3)
        try:
            dist.monitored_barrier(timeout=timedelta(seconds=3))
            q.put(("no-error", None))
        except RuntimeError as e:
            q.put(("detected", str(e)))
        q.close()
        q.join_thread()  # flush the message before leaving without teardown
        os._exit(0)
    except Exception:
        q.put(("error", traceback.format_exc()))


def test_rank_failure_is_detected_on_the_host():
    status, msg = _run(_failing_worker)
    assert status == "detected", msg
    assert "1" in msg  # names the rank that did not arrive
