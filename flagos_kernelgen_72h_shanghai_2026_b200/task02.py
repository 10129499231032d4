"""Host-side mirror of the reference operator for Task 02.

``dsa_topk_page_table_transform`` keeps the competition signature of
src/task02_dsa_topk_page_table_transform.py:1666 (scores, page_table, q_pos,
kv_lens, out_blocks, out_pages, block_size, top_k), writes into the caller's
``out_blocks`` / ``out_pages`` and returns those two objects (:1726).

Per row (b, h, q) of ``scores[B, H, Q, NB]`` it selects the ``top_k`` best
blocks of the row's causal prefix (:161-167): scores descending, ties by
block id ascending, -1 in slots the row cannot fill, and gathers
``page_table[b, id]`` for each selected id (:170-175). What the reference
routes by backend and shape (:1667-1726) is one kernel here
(libdsa_topk.so, C ABI include/dsa_topk.h).

Accepted beyond the reference's own shapes: fp32 / bf16 / fp16 scores, int32
or int64 index tensors, any ``top_k`` in [1, 2048] (also larger than NB) and
NB up to 16384 with NB % 4 == 0.

Errors: ``TypeError`` for a non-CUDA tensor or a dtype the kernel does not
take, ``ValueError`` for shapes and alignment, ``RuntimeError`` when a CUDA
call fails. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _topk_lib as L

try:  # C++ launch path (csrc/farq_fast.cpp); without it every call takes the ctypes path
    from . import _farq_fast as _fast
except ImportError:
    _fast = None
_T = torch.Tensor

_SCORE_DTYPES = {torch.float32: L.DTYPE_FP32, torch.bfloat16: L.DTYPE_BF16,
                 torch.float16: L.DTYPE_FP16}
_INDEX_DTYPES = {torch.int32: L.DTYPE_INT32, torch.int64: L.DTYPE_INT64}
_ARGS_SIZE = ctypes.sizeof(L.DsaTopkArgs)
_VALUE_ERRORS = {L.ERR_BAD_SHAPE, L.ERR_BAD_TOPK, L.ERR_ALIGNMENT, L.ERR_UNSUPPORTED,
                 L.ERR_NULL_POINTER}


def _tensor(name: str, t, device: torch.device | None) -> torch.device:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise TypeError(f"{name} is on {t.device}; CUDA tensors only")
    if device is not None and t.device != device:
        raise TypeError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.device


def _shape(name: str, t: torch.Tensor, shape: tuple) -> None:
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")


def _index_dtype(name: str, t: torch.Tensor) -> int:
    if t.dtype not in _INDEX_DTYPES:
        raise TypeError(f"{name} must be int32 or int64, got {t.dtype}")
    return _INDEX_DTYPES[t.dtype]


def dsa_topk_page_table_transform(scores: torch.Tensor, page_table: torch.Tensor,
                                  q_pos: torch.Tensor, kv_lens: torch.Tensor,
                                  out_blocks: torch.Tensor, out_pages: torch.Tensor,
                                  block_size: int, top_k: int):
    """Drop-in for the reference operator; returns ``(out_blocks, out_pages)``.

    scores [B, H, Q, NB] fp32/bf16/fp16; page_table [B, NB]; q_pos [B, Q];
    kv_lens [B]; out_blocks, out_pages [B, H, Q, top_k] (int32 or int64;
    out_pages has page_table's dtype). The launch is asynchronous on the
    current CUDA stream."""
    if (_fast is not None and _T is type(scores) and _T is type(page_table) and _T is type(q_pos)
            and _T is type(kv_lens) and _T is type(out_blocks) and _T is type(out_pages)):
        try:
            st = _fast.task02(scores, page_table, q_pos, kv_lens, out_blocks, out_pages,
                              block_size, top_k)
        except TypeError:  # a scalar pybind11 cannot convert: the checks below report it
            st = -1
        if st == L.OK:
            return out_blocks, out_pages
        if st > 0:
            _raise_status(st)
    dev = _tensor("scores", scores, None)
    for n, t in (("page_table", page_table), ("q_pos", q_pos), ("kv_lens", kv_lens),
                 ("out_blocks", out_blocks), ("out_pages", out_pages)):
        _tensor(n, t, dev)
    if scores.dtype not in _SCORE_DTYPES:
        raise TypeError(f"scores must be float32, bfloat16 or float16, got {scores.dtype}")
    if scores.dim() != 4:
        raise ValueError(f"scores must be [B, H, Q, NB], got {list(scores.shape)}")
    B, H, Q, NB = scores.shape
    top_k = int(top_k)
    block_size = int(block_size)
    _shape("page_table", page_table, (B, NB))
    _shape("q_pos", q_pos, (B, Q))
    _shape("kv_lens", kv_lens, (B,))
    _shape("out_blocks", out_blocks, (B, H, Q, top_k))
    _shape("out_pages", out_pages, (B, H, Q, top_k))
    idx = _index_dtype("q_pos", q_pos)
    if kv_lens.dtype != q_pos.dtype:
        raise TypeError(f"kv_lens must have q_pos's dtype {q_pos.dtype}, got {kv_lens.dtype}")
    pdt = _index_dtype("page_table", page_table)
    if out_pages.dtype != page_table.dtype:
        raise TypeError(f"out_pages must have page_table's dtype {page_table.dtype}, "
                        f"got {out_pages.dtype}")
    bdt = _index_dtype("out_blocks", out_blocks)

    a = L.DsaTopkArgs()
    a.struct_size = _ARGS_SIZE
    a.scores_dtype = _SCORE_DTYPES[scores.dtype]
    a.index_dtype = idx
    a.page_dtype = pdt
    a.blocks_dtype = bdt
    a.block_size = block_size
    a.top_k = top_k
    a.B, a.H, a.Q, a.NB = B, H, Q, NB
    a.scores = scores.data_ptr()
    a.page_table = page_table.data_ptr()
    a.q_pos = q_pos.data_ptr()
    a.kv_lens = kv_lens.data_ptr()
    a.out_blocks = out_blocks.data_ptr()
    a.out_pages = out_pages.data_ptr()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        st = L.load().dsa_topk_launch(ctypes.byref(a), ctypes.c_void_p(stream))
    if st != L.OK:
        _raise_status(st)
    return out_blocks, out_pages


def _raise_status(st: int):
    msg = f"dsa_topk_page_table_transform: {L.strerror(st)}"
    if st in _VALUE_ERRORS:
        raise ValueError(msg)
    if st == L.ERR_BAD_DTYPE:
        raise TypeError(msg)
    raise RuntimeError(msg)
