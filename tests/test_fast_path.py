"""The C++ launch path of the Python operators (csrc/farq_fast.cpp): it
loads, declines what it does not handle (CPU tensors, strided views) without
launching, and gives the same bytes as the ctypes path on the GPU."""
import numpy as np
import pytest
import torch

from flagos_kernelgen_72h_shanghai_2026_b200 import (dsa_topk_page_table_transform,
                                                     fused_add_rmsnorm_group_quant, task01, task02)
from flagos_kernelgen_72h_shanghai_2026_b200._build import build_fast_ext
from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import TopkWorkload, make_topk_inputs
from flagos_kernelgen_72h_shanghai_2026_b200.workloads import CONFIGS, alloc_outputs, make_inputs


@pytest.fixture(scope="module")
def fast():
    build_fast_ext()
    from flagos_kernelgen_72h_shanghai_2026_b200 import _farq_fast
    assert task01._fast is not None and task02._fast is not None, "C++ launch path not loaded"
    return _farq_fast


def test_declines_cpu_tensors(fast):
    w = CONFIGS[1].with_rows(4)
    x, r, g = make_inputs(w)
    ro, no, q, s = alloc_outputs(w, 4, "cpu")
    assert fast.task01(x, r, g, ro, no, q, s, w.eps, w.group_size, False) == -1
    tw = TopkWorkload("c", 1, 1, 2, 64, 8, 16)
    sc, pt, qp, kv = make_topk_inputs(tw)
    ob = torch.empty(1, 1, 2, 8, dtype=torch.int32)
    assert fast.task02(sc, pt, qp, kv, ob, ob.clone(), 16, 8) == -1


def _both_paths(fn):
    """Run fn() with the C++ launch path and with the ctypes path."""
    out_fast = fn()
    saved = (task01._fast, task02._fast)
    task01._fast = task02._fast = None
    try:
        out_ctypes = fn()
    finally:
        task01._fast, task02._fast = saved
    return out_fast, out_ctypes


@pytest.mark.gpu
@pytest.mark.parametrize("q_dtype", [torch.float8_e4m3fn, torch.int8])
def test_task01_same_bytes(cuda_dev, fast, q_dtype):
    w = CONFIGS[2].with_rows(300)
    x, r, g = (t.to(cuda_dev) for t in make_inputs(w))

    def run():
        ro, _, q, s = alloc_outputs(w, w.M, cuda_dev)
        q = torch.empty(w.M, w.D, dtype=q_dtype, device=cuda_dev)
        no = torch.empty(w.M, w.D, dtype=torch.bfloat16, device=cuda_dev)
        fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, w.eps, w.group_size)
        torch.cuda.synchronize(cuda_dev)
        return [t.cpu().view(torch.uint8) for t in (ro, no, q, s)]

    a, b = _both_paths(run)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


@pytest.mark.gpu
def test_task01_errors_match(cuda_dev, fast):
    w = CONFIGS[2].with_rows(8)
    x, r, g = (t.to(cuda_dev) for t in make_inputs(w))
    ro, no, q, s = alloc_outputs(w, w.M, cuda_dev)
    # D not a multiple of the group: declined by the C++ checks, raised by Python
    with pytest.raises(ValueError):
        fused_add_rmsnorm_group_quant(x, r, g, ro, no, q, s, w.eps, 96)
    # misaligned rows reach farq_launch: its status is raised
    xb = torch.empty(w.M * w.D + 1, dtype=x.dtype, device=cuda_dev)[1:].view(w.M, w.D)
    with pytest.raises(ValueError):
        fused_add_rmsnorm_group_quant(xb, r, g, ro, no, q, s, w.eps, w.group_size)


@pytest.mark.gpu
def test_task02_same_bytes(cuda_dev, fast):
    tw = TopkWorkload("f", 2, 2, 64, 2048, 64, 64, pos_mode="random", seed=3)
    sc, pt, qp, kv = (t.to(cuda_dev) for t in make_topk_inputs(tw))

    def run():
        ob = torch.empty(tw.B, tw.H, tw.Q, tw.top_k, dtype=torch.int32, device=cuda_dev)
        op = torch.empty_like(ob)
        dsa_topk_page_table_transform(sc, pt, qp, kv, ob, op, tw.block_size, tw.top_k)
        torch.cuda.synchronize(cuda_dev)
        return ob.cpu().numpy(), op.cpu().numpy()

    (a1, a2), (b1, b2) = _both_paths(run)
    np.testing.assert_array_equal(a1, b1)
    np.testing.assert_array_equal(a2, b2)
