"""Seeded synthetic inputs for the DSA top-k page-table transform (Task 02).

The reference ships no workloads; its NVIDIA routing names the competition
shapes (src/task02_dsa_topk_page_table_transform.py:1668-1672): fp32 scores
[B, H, Q, NB] with (B, H, Q, NB, top_k, block_size) in

  (2, 32, 512, 4096, 128, 64), (1, 32, 1024, 4096, 128, 64), (4, 16, 512, 4096, 128, 64)
  (1, 32, 512, 2048, 64, 128), (2, 16, 512, 2048, 64, 128), (1, 32, 1024, 2048, 64, 64)
  (1, 8, 128, 512, 32, 128), (2, 8, 128, 512, 32, 128), (1, 16, 256, 1024, 32, 128),
  (2, 16, 256, 1024, 64, 128)

and its kernel names call the score distribution Gaussian. The stand-in:
scores ~ N(0, 1) fp32; kv_lens[b] = NB * block_size (a full cache); the Q
queries of a batch are its last Q tokens, q_pos[b, q] = kv_len - Q + q, so
nearly every row has all NB blocks as candidates (the report's worst case,
R * (4 NB + 12 K) bytes, reports/task02…md). page_table[b, i] is a random
permutation of physical pages per batch.

Test-only variants add rows with negative positions, short caches, -inf
scores, exact ties (scores rounded to multiples of 1/4) and signed zeros.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class TopkWorkload:
    name: str
    B: int
    H: int
    Q: int
    NB: int
    top_k: int
    block_size: int
    dtype: torch.dtype = torch.float32
    pos_mode: str = "suffix"      # "suffix": last Q tokens; "random": uniform positions
    neg_pos_frac: float = 0.0     # fraction of queries with q_pos = -1
    short_kv: bool = False        # batch b > 0 has a cache of a random length
    ninf_frac: float = 0.0        # fraction of scores set to -inf
    tie_step: float = 0.0         # round scores to multiples of this (exact ties)
    signed_zeros: bool = False    # some scores +0.0 / -0.0
    seed: int = 0

    @property
    def rows(self) -> int:
        return self.B * self.H * self.Q

    def with_(self, **kw) -> "TopkWorkload":
        return replace(self, **kw)


TOPK_CONFIGS: dict[str, TopkWorkload] = {
    # the largest fp32 shape of the routing table: 32768 rows x 4096 blocks
    "t2_nb4096_k128_2x32x512": TopkWorkload("t2_nb4096_k128_2x32x512", 2, 32, 512, 4096, 128, 64),
    "t2_nb4096_k128_1x32x1024": TopkWorkload("t2_nb4096_k128_1x32x1024", 1, 32, 1024, 4096, 128,
                                             64),
    "t2_nb2048_k64_1x32x1024": TopkWorkload("t2_nb2048_k64_1x32x1024", 1, 32, 1024, 2048, 64, 64),
    "t2_nb2048_k64_2x16x512": TopkWorkload("t2_nb2048_k64_2x16x512", 2, 16, 512, 2048, 64, 128),
    "t2_nb1024_k64_2x16x256": TopkWorkload("t2_nb1024_k64_2x16x256", 2, 16, 256, 1024, 64, 128),
    "t2_nb512_k32_2x8x128": TopkWorkload("t2_nb512_k32_2x8x128", 2, 8, 128, 512, 32, 128),
}


def make_topk_inputs(w: TopkWorkload, device: str | torch.device = "cpu"):
    """(scores, page_table, q_pos, kv_lens) for ``w``; drawn on the CPU from
    ``torch.Generator().manual_seed(w.seed)`` in that order (so identical on
    every machine with this torch build), then moved to ``device``."""
    g = torch.Generator().manual_seed(w.seed)
    B, H, Q, NB, BS = w.B, w.H, w.Q, w.NB, w.block_size
    scores = torch.randn(B, H, Q, NB, generator=g)
    page_table = torch.stack([torch.randperm(NB * 4, generator=g)[:NB] for _ in range(B)])
    page_table = page_table.to(torch.int32)
    kv = torch.full((B,), NB * BS, dtype=torch.int64)
    if w.short_kv and B > 1:
        kv[1:] = torch.randint(0, NB * BS + 1, (B - 1,), generator=g)
    if w.pos_mode == "suffix":
        q_pos = (kv[:, None] - Q + torch.arange(Q)[None, :]).clamp(min=0)
    else:
        q_pos = torch.randint(0, NB * BS, (B, Q), generator=g)
    if w.neg_pos_frac:
        neg = torch.rand(B, Q, generator=g) < w.neg_pos_frac
        q_pos = torch.where(neg, torch.full_like(q_pos, -1), q_pos)
    if w.tie_step:
        scores = torch.round(scores / w.tie_step) * w.tie_step
    if w.signed_zeros:
        z = torch.rand(B, H, Q, NB, generator=g) < 0.05
        sign = torch.rand(B, H, Q, NB, generator=g) < 0.5
        scores = torch.where(z, torch.where(sign, -0.0, 0.0), scores)
    if w.ninf_frac:
        m = torch.rand(B, H, Q, NB, generator=g) < w.ninf_frac
        scores = scores.masked_fill(m, float("-inf"))
    scores = scores.to(w.dtype)
    dev = torch.device(device)
    return (scores.to(dev), page_table.to(dev), q_pos.to(torch.int32).to(dev),
            kv.to(torch.int32).to(dev))


def topk_bytes_per_call(w: TopkWorkload, n_candidates: torch.Tensor | None = None) -> int:
    """Algorithmic HBM bytes of one call: every candidate score read once
    (the causal prefix of each row), q_pos / kv_lens once per row, and per
    output slot a 4-byte block id, a 4-byte page written and a 4-byte page
    entry read (the report's 12 K per row). Without ``n_candidates`` every
    row is taken as fully valid: R * (d * NB + 12 K)."""
    d = torch.tensor([], dtype=w.dtype).element_size()
    R = w.rows
    cand = R * w.NB if n_candidates is None else int(n_candidates.sum())
    return d * cand + R * 12 * w.top_k + R * 8
