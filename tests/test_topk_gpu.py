"""Task 02 on the GPU: libdsa_topk.so against the reference's own outputs
(golden fixtures) and against the oracle, bit-exact (ids and pages are
integers), at the reference's competition shapes and at the edges of the
kernel's range."""
import numpy as np
import pytest
import torch

from topk_cases import TOPK_CASES, topk_case_inputs
from pathlib import Path

from oracle.dsa_topk_oracle import dsa_topk_page_table_transform_ref
from flagos_kernelgen_72h_shanghai_2026_b200 import dsa_topk_page_table_transform
from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import (
    TOPK_CONFIGS, TopkWorkload, make_topk_inputs)

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on CPU-only hosts)")
    from flagos_kernelgen_72h_shanghai_2026_b200._build import build_topk_lib
    build_topk_lib()
    return torch.device("cuda:0")


def run(dev, w, s, pt, qp, kv, blocks_dtype=torch.int32, page_dtype=None, index_dtype=None):
    pt = pt.to(page_dtype) if page_dtype is not None else pt
    if index_dtype is not None:
        qp, kv = qp.to(index_dtype), kv.to(index_dtype)
    sd, ptd, qpd, kvd = (t.to(dev) for t in (s, pt, qp, kv))
    ob = torch.full((w.B, w.H, w.Q, w.top_k), 7, dtype=blocks_dtype, device=dev)
    op = torch.full((w.B, w.H, w.Q, w.top_k), 7, dtype=ptd.dtype, device=dev)
    out = dsa_topk_page_table_transform(sd, ptd, qpd, kvd, ob, op, w.block_size, w.top_k)
    assert out[0] is ob and out[1] is op
    torch.cuda.synchronize(dev)
    return ob.cpu().to(torch.int64).numpy(), op.cpu().to(torch.int64).numpy()


def check_vs_oracle(dev, w, **kw):
    s, pt, qp, kv = make_topk_inputs(w)
    ob, op = run(dev, w, s, pt, qp, kv, **kw)
    rb, rp = dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    mism = int((ob != rb).sum())
    assert mism == 0, f"{mism} block ids differ from the oracle"
    assert int((op != rp).sum()) == 0, "pages differ from the oracle"
    return s, ob


@pytest.mark.parametrize("name", sorted(TOPK_CASES))
def test_golden_reference_outputs(dev, name):
    d = np.load(GOLDEN / f"topk_{name}.npz")
    w, s, pt, qp, kv = topk_case_inputs(name)
    ob, op = run(dev, w, s, pt, qp, kv)
    np.testing.assert_array_equal(ob, d["out_blocks"].astype(np.int64))
    np.testing.assert_array_equal(op, d["out_pages"].astype(np.int64))


@pytest.mark.parametrize("name", sorted(TOPK_CONFIGS))
def test_competition_shapes_vs_oracle(dev, name):
    s, ob = check_vs_oracle(dev, TOPK_CONFIGS[name])
    # size-independent properties: ids unique per row, scores non-increasing
    B, H, Q, K = ob.shape
    rows = ob.reshape(-1, K)
    sc = s.float().reshape(-1, s.shape[-1]).numpy()
    pick = np.take_along_axis(sc, np.maximum(rows, 0), axis=1)
    assert (np.diff(pick, axis=1)[rows[:, 1:] >= 0] <= 0).all()


@pytest.mark.parametrize("w", [
    # every dtype and launch shape (T = 128 / 256 / 512, J = 1..8)
    TopkWorkload("e_bf16_nb4096", 1, 4, 64, 4096, 128, 64, dtype=torch.bfloat16, seed=31),
    TopkWorkload("e_fp16_nb2048", 1, 4, 64, 2048, 64, 64, dtype=torch.float16, seed=32),
    TopkWorkload("e_nb16384_k2048", 1, 2, 8, 16384, 2048, 16, pos_mode="random", seed=33),
    TopkWorkload("e_nb12288_k512", 1, 1, 16, 12288, 512, 64, seed=34),
    TopkWorkload("e_nb8192_bf16", 2, 1, 16, 8192, 256, 32, dtype=torch.bfloat16, seed=35),
    TopkWorkload("e_nb1536", 1, 2, 16, 1536, 100, 8, pos_mode="random", seed=36),
    TopkWorkload("e_nb4", 3, 2, 5, 4, 3, 2, pos_mode="random", short_kv=True, seed=37),
    TopkWorkload("e_nb20_k32", 2, 2, 5, 20, 32, 3, pos_mode="random", seed=38),
    # K larger than the row, K = 1
    TopkWorkload("e_k_gt_nb", 1, 2, 8, 256, 300, 4, seed=39),
    TopkWorkload("e_k1", 2, 2, 32, 1024, 1, 64, pos_mode="random", seed=40),
    # masks: negative positions, short and empty caches, -inf, signed zeros
    TopkWorkload("e_masks", 4, 2, 32, 1024, 64, 16, pos_mode="random", neg_pos_frac=0.2,
                 short_kv=True, ninf_frac=0.5, signed_zeros=True, seed=41),
    TopkWorkload("e_all_ninf", 1, 1, 8, 512, 32, 8, ninf_frac=1.0, seed=42),
    # heavy ties (keys equal across the K-th boundary: the id tie-break)
    TopkWorkload("e_ties_coarse", 1, 2, 16, 4096, 128, 64, tie_step=2.0, seed=43),
    TopkWorkload("e_ties_bf16", 1, 2, 16, 2048, 64, 64, dtype=torch.bfloat16, tie_step=1.0,
                 seed=44),
], ids=lambda w: w.name)
def test_edges_vs_oracle(dev, w):
    check_vs_oracle(dev, w)


def test_constant_scores_pick_lowest_ids(dev):
    w = TopkWorkload("const", 1, 1, 4, 4096, 128, 64)
    s, pt, qp, kv = make_topk_inputs(w)
    s = torch.full_like(s, 0.5)
    ob, op = run(dev, w, s, pt, qp, kv)
    np.testing.assert_array_equal(ob[0, 0, 0], np.arange(128))


def test_nan_scores_follow_the_key_order(dev):
    w = TopkWorkload("nan", 1, 2, 8, 1024, 64, 64, seed=45)
    s, pt, qp, kv = make_topk_inputs(w)
    flat = s.view(-1)
    flat[::97] = float("nan")
    flat.view(torch.int32)[5::193] = -1  # the all-ones NaN pattern (key 0: never selected)
    ob, op = run(dev, w, s, pt, qp, kv)
    rb, rp = dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    np.testing.assert_array_equal(ob, rb)
    np.testing.assert_array_equal(op, rp)


@pytest.mark.parametrize("dtypes", [
    dict(blocks_dtype=torch.int64, page_dtype=torch.int64, index_dtype=torch.int64),
    dict(blocks_dtype=torch.int64, page_dtype=torch.int32, index_dtype=torch.int32),
    dict(blocks_dtype=torch.int32, page_dtype=torch.int64, index_dtype=torch.int64),
], ids=["all64", "blocks64", "pages64"])
def test_index_dtypes(dev, dtypes):
    check_vs_oracle(dev, TopkWorkload("idx", 2, 2, 16, 2048, 64, 128, pos_mode="random", seed=46),
                    **dtypes)


def test_side_stream_and_graph_replay(dev):
    w = TopkWorkload("g", 1, 4, 64, 4096, 128, 64, seed=47)
    s, pt, qp, kv = make_topk_inputs(w)
    rb, rp = dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    sd, ptd, qpd, kvd = (t.to(dev) for t in (s, pt, qp, kv))
    ob = torch.empty(w.B, w.H, w.Q, w.top_k, dtype=torch.int32, device=dev)
    op = torch.empty_like(ob)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        dsa_topk_page_table_transform(sd, ptd, qpd, kvd, ob, op, w.block_size, w.top_k)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            dsa_topk_page_table_transform(sd, ptd, qpd, kvd, ob, op, w.block_size, w.top_k)
    ob.fill_(-7)
    op.fill_(-7)
    g.replay()
    torch.cuda.synchronize(dev)
    np.testing.assert_array_equal(ob.cpu().numpy(), rb)
    np.testing.assert_array_equal(op.cpu().numpy(), rp)


def test_wrapper_errors(dev):
    w = TopkWorkload("err", 1, 1, 2, 64, 8, 16)
    s, pt, qp, kv = (t.to(dev) for t in make_topk_inputs(w))
    ob = torch.empty(1, 1, 2, 8, dtype=torch.int32, device=dev)
    with pytest.raises(ValueError):
        dsa_topk_page_table_transform(s, pt, qp, kv, ob[..., :4], ob.clone(), 16, 8)
    with pytest.raises(TypeError):
        dsa_topk_page_table_transform(s.to(torch.float64), pt, qp, kv, ob, ob.clone(), 16, 8)
    with pytest.raises(ValueError):
        dsa_topk_page_table_transform(s[..., :62].contiguous(), pt[:, :62].contiguous(), qp, kv,
                                      ob, ob.clone(), 16, 8)
