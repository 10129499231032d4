"""CPU oracle for Task 02, the DSA top-k page-table transform (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker or the timed CPU baseline. The product path never
imports it.

Restates sinpeyw/flagos-kernelgen-72h-shanghai-2026,
src/task02_dsa_topk_page_table_transform.py (``T2`` below):

* Row r = (b, h, q) of scores[B, H, Q, NB] (row-major, offset r*NB + block;
  T2:157-160, :164).
* Causal prefix (T2:161-166): pos = q_pos[b*Q + q], kv = kv_lens[b], both
  cast to int32; valid_blocks = min(ceil(kv / block_size), NB);
  last = min(pos // block_size, valid_blocks - 1); block i is a candidate iff
  pos >= 0 and i <= last.
* A candidate is selectable iff its score (cast to fp32) is not -inf
  (T2:166-167, :539).
* Order (T2:489-505, the packed key of the NVIDIA paths): the score mapped to
  an order-preserving 32-bit key (-0.0 folded to +0.0 first; negative values
  bit-inverted, others with the sign bit set), then the block id ascending
  (the key's low word is 0xFFFFFFFF - id, larger first).
* out_blocks[r, k] = id of the k-th best selectable block, -1 when the row has
  fewer than k+1 (T2:170-175, :507-517); out_pages[r, k] =
  page_table[b*NB + id] (page_table row-major [B, NB]), -1 likewise.
* A selectable element whose key is 0 (only the all-ones NaN bit pattern)
  has no value in the reference's unpacking (``ordered_score != 0``,
  T2:513-516) and ranks below every other element, so it can only occupy an
  output slot that is -1 anyway: it is treated as not selectable.

The report's statement of the contract (reports/task02…md): scores descending,
ties by block id ascending, invalid slots -1, page gather by the selected id.

Parity note: the reference's NVIDIA routes for NB in {1024, 2048} with K=64
and for the chunked NB >= 2048 paths first select with a 32-bit code whose
low log2(chunk or NB) bits are replaced by the block id (T2:567-571,
:621-632), then re-rank exactly. Two scores that agree in all but those low
key bits are ordered by id there, so at a chunk's K-th boundary the
reference can keep the lower-scored of two near-equal elements. This oracle
follows the stated contract (exact order); tests/golden records where the
reference's own output differs from it.
"""
from __future__ import annotations

import numpy as np


def ordered_keys(scores_f32: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 key of fp32 scores (T2:489-494)."""
    x = np.where(scores_f32 == 0.0, np.float32(0.0), scores_f32).astype(np.float32)
    bits = x.view(np.uint32)
    neg = (bits >> np.uint32(31)) != 0
    return np.where(neg, ~bits, bits ^ np.uint32(0x80000000)).astype(np.uint32)


def candidate_counts(q_pos: np.ndarray, kv_lens: np.ndarray, B: int, H: int, Q: int, NB: int,
                     block_size: int) -> np.ndarray:
    """Number of leading candidate blocks of every row [B*H*Q] (T2:161-166)."""
    pos = np.asarray(q_pos).reshape(B, Q).astype(np.int64).astype(np.int32).astype(np.int64)
    kv = np.asarray(kv_lens).reshape(B).astype(np.int64).astype(np.int32).astype(np.int64)
    valid_blocks = np.minimum(-(-kv // block_size), NB)          # ceil for kv >= 0
    valid_blocks = np.where(kv > 0, valid_blocks, 0)              # kv <= 0: nothing valid
    last = np.minimum(np.floor_divide(pos, block_size), (valid_blocks - 1)[:, None])
    n = np.where(pos >= 0, np.maximum(last + 1, 0), 0)           # [B, Q]
    return np.broadcast_to(n[:, None, :], (B, H, Q)).reshape(-1)


def dsa_topk_page_table_transform_ref(scores, page_table, q_pos, kv_lens, block_size: int,
                                      top_k: int):
    """Returns (out_blocks [B,H,Q,K] int64, out_pages [B,H,Q,K] int64) for
    CPU tensors or numpy arrays (scores any float dtype, page_table [B, NB])."""
    import torch
    if isinstance(scores, torch.Tensor):
        scores = scores.float().numpy()
    if isinstance(page_table, torch.Tensor):
        page_table = page_table.numpy()
    if isinstance(q_pos, torch.Tensor):
        q_pos = q_pos.numpy()
    if isinstance(kv_lens, torch.Tensor):
        kv_lens = kv_lens.numpy()
    B, H, Q, NB = scores.shape
    R = B * H * Q
    K = int(top_k)
    s = np.asarray(scores, dtype=np.float32).reshape(R, NB)
    n = candidate_counts(q_pos, kv_lens, B, H, Q, NB, block_size)
    key = ordered_keys(s).astype(np.uint64)
    ids = np.arange(NB, dtype=np.uint64)
    packed = (key << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids)[None, :]
    selectable = (np.arange(NB)[None, :] < n[:, None]) & (s != -np.inf) & (key != 0)
    packed = np.where(selectable, packed, np.uint64(0))
    # descending order of the packed keys: every selectable key is unique
    # (distinct ids), unselectable ones are 0 and sort last
    kk = min(K, NB)
    if kk < NB:
        part = np.argpartition(~packed, kk - 1, axis=1)[:, :kk]
    else:
        part = np.broadcast_to(np.arange(NB)[None, :], (R, NB))
    sel_keys = np.take_along_axis(packed, part, axis=1)
    order = np.argsort(~sel_keys, axis=1, kind="stable")
    best = np.take_along_axis(sel_keys, order, axis=1)
    blocks = (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)
    has = best != 0
    blocks = np.where(has, blocks, -1)
    out_blocks = np.full((R, K), -1, dtype=np.int64)
    out_blocks[:, :kk] = blocks
    batch = np.arange(R) // (H * Q)
    pt = np.asarray(page_table).reshape(B, NB).astype(np.int64)
    pages = np.where(out_blocks >= 0, pt[batch[:, None], np.maximum(out_blocks, 0)], -1)
    return out_blocks.reshape(B, H, Q, K), pages.reshape(B, H, Q, K)
