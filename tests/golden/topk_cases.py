"""Golden cases of the DSA top-k page-table transform (Task 02): shapes and
seeded inputs shared by make_golden_topk.py (which runs the reference's own
kernels once, in this repository's build container) and the tests (which
regenerate the same inputs, check their digest and compare with the stored
outputs). Each case names the reference route its shape takes on an NVIDIA
device (src/task02_dsa_topk_page_table_transform.py:1666-1726, :771-817).
"""
from __future__ import annotations

import hashlib

import torch

from flagos_kernelgen_72h_shanghai_2026_b200.topk_workloads import TopkWorkload, make_topk_inputs

W = TopkWorkload
# name -> (workload, reference route)
TOPK_CASES = {
    "single_nb512_k32_bs128": (
        W("tg1", 2, 2, 4, 512, 32, 128, pos_mode="random", seed=11),
        "_packed_single_gather_kernel (CHUNK_N=512)"),
    "single_nb1024_k32": (
        W("tg2", 1, 2, 4, 1024, 32, 64, pos_mode="random", seed=12),
        "_packed_single_gather_kernel (CHUNK_N=1024)"),
    "prefix_nb1024_k64": (
        W("tg3", 1, 2, 4, 1024, 64, 64, seed=13),
        "_packed_prefix_single_gather_kernel"),
    "prefix_nb2048_k64_bf16": (
        W("tg4", 1, 1, 4, 2048, 64, 128, dtype=torch.bfloat16, seed=14),
        "_packed_prefix_single_gather_kernel"),
    "chunked_nb4096_k128": (
        W("tg5", 1, 1, 6, 4096, 128, 64, seed=15),
        "_packed_local_select_kernel (8 x 512) + _legacy_u64_sort_merge_ids_gather_kernel"),
    "chunked_nb2048_k128_random_pos": (
        W("tg6", 2, 1, 3, 2048, 128, 64, pos_mode="random", seed=16),
        "_packed_local_select_kernel (4 x 512) + _legacy_u64_sort_merge_ids_gather_kernel"),
    "edges_nb512_k64": (
        W("tg7", 3, 2, 4, 512, 64, 16, pos_mode="random", neg_pos_frac=0.25, short_kv=True,
          ninf_frac=0.3, signed_zeros=True, seed=17),
        "_packed_single_gather_kernel (CHUNK_N=512)"),
    "ties_nb4096_k128": (
        W("tg8", 1, 1, 4, 4096, 128, 64, tie_step=0.25, seed=18),
        "_packed_local_select_kernel (8 x 512) + _legacy_u64_sort_merge_ids_gather_kernel"),
    "ties_fp16_nb1024_k64": (
        W("tg9", 1, 2, 3, 1024, 64, 32, dtype=torch.float16, tie_step=0.5, pos_mode="random",
          seed=19),
        "_packed_prefix_single_gather_kernel"),
}


def topk_case_inputs(name: str):
    """(workload, scores, page_table, q_pos, kv_lens) on CPU for a golden case."""
    w, _ = TOPK_CASES[name]
    return (w,) + make_topk_inputs(w)


def topk_input_digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()
