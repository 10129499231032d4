"""Host-buffer entry point: the same operator on tensors that live in host memory.

``fused_add_rmsnorm_group_quant_host`` takes x, residual and the four output
tensors on the CPU (pinned memory for asynchronous copies) and streams them
through the GPU in row chunks: chunk i+1 is copied host->device while chunk i
runs the kernel and chunk i-1 is copied device->host, on three CUDA streams
ordered by events. PCIe carries both directions at once, so a call costs about
the larger of its two transfer volumes rather than their sum.

The reference has no host-memory path; this is an extension for callers that
keep activations on the host. Each chunk is processed by the same sm_100a
kernel as the device entry point (no CPU compute).

The call returns once the work is queued. The caller's current stream is made
to wait for the last copy, so ``torch.cuda.current_stream().synchronize()``
(or any later work on that stream) sees complete outputs.
"""
from __future__ import annotations

import torch

from .task01 import fused_add_rmsnorm_group_quant

_SLOTS = 3


class _Pipeline:
    """Device staging buffers, streams and events of one (device, shape) pipeline."""

    def __init__(self, device, chunk, D, groups, x_dtype, rout_dtype, norm_dtype, q_dtype):
        self.device = device
        mk = lambda shape, dt: torch.empty(shape, dtype=dt, device=device)  # noqa: E731
        self.slots = []
        for _ in range(_SLOTS):
            self.slots.append(dict(
                x=mk((chunk, D), x_dtype), r=mk((chunk, D), x_dtype),
                ro=mk((chunk, D), rout_dtype),
                no=mk((chunk, D), norm_dtype) if norm_dtype is not None else None,
                q=mk((chunk, D), q_dtype), s=mk((chunk, groups), torch.float32)))
        self.h2d = torch.cuda.Stream(device)
        self.comp = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        ev = lambda: torch.cuda.Event()  # noqa: E731
        self.ev_in = [ev() for _ in range(_SLOTS)]
        self.ev_done = [ev() for _ in range(_SLOTS)]
        self.ev_out = [ev() for _ in range(_SLOTS)]
        self.used = [False] * _SLOTS


_PIPES: dict = {}     # (device, shape, dtypes) -> _Pipeline, least recently used first
_MAX_PIPES = 4        # staging buffers kept alive for at most this many shapes


def fused_add_rmsnorm_group_quant_host(x, residual, gamma, residual_out, norm_out, x_q, x_scale,
                                       eps, group_size, *, ue8m0=False, device=None,
                                       chunk_rows=512):
    """Same contract as ``fused_add_rmsnorm_group_quant`` for host tensors
    (x, residual, residual_out, norm_out, x_q, x_scale on the CPU; gamma on
    the CPU or on ``device``). Returns the same four objects."""
    device = torch.device(device if device is not None else "cuda")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    for name, t in (("x", x), ("residual", residual), ("residual_out", residual_out),
                    ("x_q", x_q), ("x_scale", x_scale)):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise TypeError(f"{name} must be a CPU tensor for the host-buffer entry point")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, D], got {list(x.shape)}")
    M, D = x.shape
    write_norm = norm_out is not None and norm_out.numel() > 0
    if M == 0:
        return residual_out, norm_out, x_q, x_scale
    chunk = max(1, min(int(chunk_rows), M))
    groups = D // int(group_size) if group_size else 0
    key = (device, chunk, D, groups, x.dtype, residual_out.dtype,
           norm_out.dtype if write_norm else None, x_q.dtype)
    pipe = _PIPES.pop(key, None)
    if pipe is None:
        if len(_PIPES) >= _MAX_PIPES:
            old = _PIPES.pop(next(iter(_PIPES)))
            old.d2h.synchronize()  # its last copies have finished with its buffers
        pipe = _Pipeline(device, chunk, D, groups, x.dtype, residual_out.dtype,
                         norm_out.dtype if write_norm else None, x_q.dtype)
    _PIPES[key] = pipe  # most recently used last
    g = gamma.to(device, non_blocking=True) if gamma.device != device else gamma
    caller = torch.cuda.current_stream(device)
    ev_start = torch.cuda.Event()
    ev_start.record(caller)
    for st in (pipe.h2d, pipe.comp, pipe.d2h):
        st.wait_event(ev_start)  # gamma copy and earlier caller work first

    for i, a in enumerate(range(0, M, chunk)):
        b = min(M, a + chunk)
        n = b - a
        k = i % _SLOTS
        sl = pipe.slots[k]
        with torch.cuda.stream(pipe.h2d):
            if pipe.used[k]:
                pipe.h2d.wait_event(pipe.ev_out[k])  # previous user of the slot copied out
            sl["x"][:n].copy_(x[a:b], non_blocking=True)
            sl["r"][:n].copy_(residual[a:b], non_blocking=True)
            pipe.ev_in[k].record(pipe.h2d)
        with torch.cuda.stream(pipe.comp):
            pipe.comp.wait_event(pipe.ev_in[k])
            fused_add_rmsnorm_group_quant(
                sl["x"][:n], sl["r"][:n], g, sl["ro"][:n],
                sl["no"][:n] if write_norm else None, sl["q"][:n], sl["s"][:n],
                eps, group_size, ue8m0=ue8m0)
            pipe.ev_done[k].record(pipe.comp)
        with torch.cuda.stream(pipe.d2h):
            pipe.d2h.wait_event(pipe.ev_done[k])
            residual_out[a:b].copy_(sl["ro"][:n], non_blocking=True)
            if write_norm:
                norm_out[a:b].copy_(sl["no"][:n], non_blocking=True)
            x_q[a:b].copy_(sl["q"][:n], non_blocking=True)
            x_scale[a:b].copy_(sl["s"][:n], non_blocking=True)
            pipe.ev_out[k].record(pipe.d2h)
        pipe.used[k] = True
    if g is not gamma:
        # gamma was copied to the device for this call: keep that copy alive
        # until the kernels on the pipeline's compute stream have read it
        g.record_stream(pipe.comp)
    last = torch.cuda.Event()
    last.record(pipe.d2h)
    caller.wait_event(last)
    return residual_out, norm_out, x_q, x_scale
