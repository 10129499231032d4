"""Task 02 (DSA top-k page-table transform) without a GPU: the oracle against
the reference's own outputs (golden fixtures made by running the reference's
kernels, tests/golden/make_golden_topk.py) and against a brute-force
restatement of the contract; libdsa_topk.so loads, exports every entry point
include/dsa_topk.h declares and answers bad arguments with status codes
before any device work."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from topk_cases import TOPK_CASES, topk_case_inputs, topk_input_digest
from oracle.dsa_topk_oracle import candidate_counts, dsa_topk_page_table_transform_ref, ordered_keys
from flagos_kernelgen_72h_shanghai_2026_b200 import _topk_lib as L
from flagos_kernelgen_72h_shanghai_2026_b200._build import TOPK_LIB_PATH, build_topk_lib
from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import TopkWorkload, make_topk_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"
HEADER = Path(__file__).resolve().parent.parent / "include" / "dsa_topk.h"


@pytest.mark.parametrize("name", sorted(TOPK_CASES))
def test_oracle_matches_reference_golden(name):
    path = GOLDEN / f"topk_{name}.npz"
    if not path.exists():
        pytest.fail(f"missing fixture {path.name}: run tests/golden/make_golden_topk.py")
    d = np.load(path)
    w, s, pt, qp, kv = topk_case_inputs(name)
    assert topk_input_digest(s, pt, qp, kv) == str(d["digest"]), "inputs differ from the fixture's"
    ob, op = dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    np.testing.assert_array_equal(ob, d["out_blocks"].astype(np.int64))
    np.testing.assert_array_equal(op, d["out_pages"].astype(np.int64))


def brute_force(scores, page_table, q_pos, kv_lens, block_size, top_k):
    """The contract stated row by row with Python sorting (small cases only)."""
    B, H, Q, NB = scores.shape
    s = scores.float()
    ob = np.full((B, H, Q, top_k), -1, dtype=np.int64)
    op = np.full((B, H, Q, top_k), -1, dtype=np.int64)
    for b in range(B):
        kv = int(kv_lens[b])
        valid = min(-(-kv // block_size), NB) if kv > 0 else 0
        for q in range(Q):
            pos = int(q_pos[b, q])
            last = min(pos // block_size, valid - 1) if pos >= 0 else -1
            for h in range(H):
                cand = []
                for i in range(last + 1):
                    v = float(s[b, h, q, i])
                    if v == float("-inf") or np.isnan(v) and ordered_keys(
                            np.array([v], np.float32))[0] == 0:
                        continue
                    k = int(ordered_keys(np.array([v], np.float32))[0])
                    cand.append((-k, i))
                cand.sort()
                for j, (_, i) in enumerate(cand[:top_k]):
                    ob[b, h, q, j] = i
                    op[b, h, q, j] = int(page_table[b, i])
    return ob, op


@pytest.mark.parametrize("w", [
    TopkWorkload("bf1", 2, 2, 3, 64, 8, 16, pos_mode="random", neg_pos_frac=0.3, short_kv=True,
                 ninf_frac=0.2, signed_zeros=True, seed=1),
    TopkWorkload("bf2", 1, 1, 4, 32, 40, 4, tie_step=0.5, pos_mode="random", seed=2),
    TopkWorkload("bf3", 2, 1, 2, 128, 16, 8, dtype=torch.bfloat16, tie_step=0.25, seed=3),
    TopkWorkload("bf4", 3, 1, 2, 16, 4, 1, dtype=torch.float16, short_kv=True, seed=4),
], ids=lambda w: w.name)
def test_oracle_matches_brute_force(w):
    s, pt, qp, kv = make_topk_inputs(w)
    ob, op = dsa_topk_page_table_transform_ref(s, pt, qp, kv, w.block_size, w.top_k)
    rb, rp = brute_force(s, pt, qp, kv, w.block_size, w.top_k)
    np.testing.assert_array_equal(ob, rb)
    np.testing.assert_array_equal(op, rp)


def test_ordered_keys_order_and_signed_zero():
    v = np.array([-np.inf, -3.0, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], dtype=np.float32)
    k = ordered_keys(v)
    assert k[3] == k[4]
    assert all(int(a) < int(b) for a, b in zip(k[:3], k[1:4]))
    assert all(int(a) < int(b) for a, b in zip(k[4:], k[5:]))


def test_candidate_counts_rules():
    # pos // bs against min(ceil(kv / bs), NB) - 1; negative pos or empty cache -> 0
    q_pos = np.array([[-1, 0, 63, 64, 10_000]], dtype=np.int32)
    n = candidate_counts(q_pos, np.array([130], np.int32), 1, 1, 5, 8, 64)
    assert n.tolist() == [0, 1, 1, 2, 3]
    n = candidate_counts(q_pos, np.array([0], np.int32), 1, 1, 5, 8, 64)
    assert n.tolist() == [0, 0, 0, 0, 0]


# ------------------------------------------------------------- C ABI
@pytest.fixture(scope="module")
def lib():
    build_topk_lib()
    return L.load()


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return re.findall(r"^\s*(?:int|const char\*)\s+(dsa_topk_\w+)\s*\(", text, flags=re.M)


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert {"dsa_topk_launch", "dsa_topk_strerror", "dsa_topk_abi_version"} <= set(names)
    raw = ctypes.CDLL(str(TOPK_LIB_PATH))
    for name in names:
        assert hasattr(raw, name), f"{name} declared in dsa_topk.h but not exported"


def test_struct_layout(lib):
    assert ctypes.sizeof(L.DsaTopkArgs) == 8 * 4 + 4 * 8 + 6 * 8
    assert lib.dsa_topk_abi_version() == L.ABI_VERSION
    for code in range(0, 9):
        assert lib.dsa_topk_strerror(code)
    assert b"unknown" in lib.dsa_topk_strerror(99)


def _args(**kw):
    a = L.DsaTopkArgs()
    a.struct_size = ctypes.sizeof(a)
    a.scores_dtype, a.index_dtype, a.page_dtype, a.blocks_dtype = (
        L.DTYPE_FP32, L.DTYPE_INT32, L.DTYPE_INT32, L.DTYPE_INT32)
    a.block_size, a.top_k = 64, 128
    a.B, a.H, a.Q, a.NB = 1, 1, 1, 4096
    for i, f in enumerate(("scores", "page_table", "q_pos", "kv_lens", "out_blocks", "out_pages")):
        setattr(a, f, 0x10000 * (i + 1))  # never dereferenced: every case fails validation
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    (dict(struct_size=8), L.ERR_BAD_ARGS_SIZE),
    (dict(reserved0=1), L.ERR_BAD_ARGS_SIZE),
    (dict(NB=4094), L.ERR_BAD_SHAPE),
    (dict(NB=0), L.ERR_BAD_SHAPE),
    (dict(B=-1), L.ERR_BAD_SHAPE),
    (dict(block_size=0), L.ERR_BAD_SHAPE),
    (dict(top_k=0), L.ERR_BAD_TOPK),
    (dict(top_k=4096), L.ERR_BAD_TOPK),
    (dict(scores_dtype=L.DTYPE_INT32), L.ERR_BAD_DTYPE),
    (dict(index_dtype=L.DTYPE_FP32), L.ERR_BAD_DTYPE),
    (dict(page_dtype=7), L.ERR_BAD_DTYPE),
    (dict(NB=32768), L.ERR_UNSUPPORTED),
    (dict(B=1 << 30, H=1 << 30, Q=1 << 30), L.ERR_BAD_SHAPE),
    (dict(B=1 << 16, H=1 << 15, Q=1, NB=4), L.ERR_UNSUPPORTED),
    (dict(scores=0), L.ERR_NULL_POINTER),
    (dict(out_pages=0), L.ERR_NULL_POINTER),
    (dict(scores=0x10008), L.ERR_ALIGNMENT),
    (dict(page_dtype=L.DTYPE_INT64, page_table=0x10004), L.ERR_ALIGNMENT),
    (dict(q_pos=0x10002), L.ERR_ALIGNMENT),
])
def test_validation_before_any_device_call(lib, kw, code):
    assert lib.dsa_topk_launch(ctypes.byref(_args(**kw)), None) == code


def test_empty_rows_are_a_no_op(lib):
    assert lib.dsa_topk_launch(ctypes.byref(_args(Q=0)), None) == L.OK
    assert lib.dsa_topk_launch(ctypes.byref(_args(B=0, scores=0)), None) == L.OK


def test_wrapper_rejects_cpu_tensors():
    from flagos_kernelgen_72h_shanghai_2026_b200 import dsa_topk_page_table_transform
    w = TopkWorkload("c", 1, 1, 2, 64, 8, 16)
    s, pt, qp, kv = make_topk_inputs(w)
    ob = torch.empty(1, 1, 2, 8, dtype=torch.int32)
    with pytest.raises(TypeError):
        dsa_topk_page_table_transform(s, pt, qp, kv, ob, ob.clone(), 16, 8)
