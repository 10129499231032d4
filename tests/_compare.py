"""Parity checks shared by the tests (test infrastructure).

Tolerances (from the operator's acceptance bar):
  * residual_out: bit-exact.
  * x_scale: relative error <= 1e-6 (and UE8M0 scales equal, except a
    power-of-two boundary flip on at most 1e-4 of the groups).
  * x_q: at most 1 quantisation step (int8) or 1 e4m3 ulp apart, on at
    most 0.1% of the elements.
  * norm_out: at most 1 ulp of its dtype apart, on at most 0.1% of elements.
"""
from __future__ import annotations

import torch

SCALE_RTOL = 1e-6
Q_MAX_FRAC = 1e-3
NORM_MAX_FRAC = 1e-3


def _ordered(t: torch.Tensor, nbits: int) -> torch.Tensor:
    """Map sign-magnitude float bit patterns to integers ordered like the values."""
    mag_mask = (1 << (nbits - 1)) - 1
    b = t.to(torch.int64)
    mag = b & mag_mask
    neg = (b >> (nbits - 1)) & 1
    return torch.where(neg == 1, -mag, mag)


def float_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|ulp distance| between two same-dtype float tensors (bf16/fp16/fp32)."""
    assert a.dtype == b.dtype
    if a.dtype in (torch.bfloat16, torch.float16):
        ia, ib = a.view(torch.int16).to(torch.int64) & 0xFFFF, b.view(torch.int16).to(torch.int64) & 0xFFFF
        return (_ordered(ia, 16) - _ordered(ib, 16)).abs()
    ia, ib = a.view(torch.int32).to(torch.int64) & 0xFFFFFFFF, b.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return (_ordered(ia, 32) - _ordered(ib, 32)).abs()


def q_diff(q_gpu: torch.Tensor, q_ref: torch.Tensor, mode: str) -> torch.Tensor:
    """Steps (int8) or e4m3 ulps between two quantised tensors (CPU)."""
    if mode == "int8":
        return (q_gpu.view(torch.int8).to(torch.int64) - q_ref.view(torch.int8).to(torch.int64)).abs()
    a = q_gpu.view(torch.uint8).to(torch.int64)
    b = q_ref.view(torch.uint8).to(torch.int64)
    return (_ordered(a, 8) - _ordered(b, 8)).abs()


def check_outputs(got: dict, ref: dict, mode: str, ue8m0: bool = False,
                  check_norm: bool = True) -> dict:
    """Assert parity of CPU copies of the GPU outputs against the oracle's."""
    stats = {}
    ro, rro = got["residual_out"], ref["residual_out"]
    assert ro.dtype == rro.dtype and ro.shape == rro.shape
    nbad = int((float_ulp_diff(ro, rro) != 0).sum())
    assert nbad == 0, f"residual_out not bit-exact: {nbad} elements differ"

    s, rs = got["x_scale"], ref["x_scale"]
    if ue8m0:
        flips = (s != rs)
        frac = flips.float().mean().item()
        ratio = (s[flips] / rs[flips])
        assert frac <= 1e-4 and bool(((ratio == 2) | (ratio == 0.5)).all()), \
            f"ue8m0 scales differ on {frac:.2e} of groups"
        stats["scale_flips"] = int(flips.sum())
    else:
        rel = ((s - rs).abs() / rs.abs()).max().item() if s.numel() else 0.0
        assert rel <= SCALE_RTOL, f"scale rel err {rel:.3e} > {SCALE_RTOL}"
        stats["scale_rel"] = rel

    d = q_diff(got["x_q"], ref["x_q"], mode)
    dmax = int(d.max()) if d.numel() else 0
    frac = (d != 0).float().mean().item() if d.numel() else 0.0
    assert dmax <= 1, f"q differs by {dmax} steps/ulps"
    assert frac <= Q_MAX_FRAC, f"q differs on {frac:.3e} of elements"
    stats["q_mismatch_frac"] = frac

    if check_norm and got.get("norm_out") is not None:
        nd = float_ulp_diff(got["norm_out"], ref["norm_out"])
        nmax = int(nd.max()) if nd.numel() else 0
        nfrac = (nd != 0).float().mean().item() if nd.numel() else 0.0
        assert nmax <= 1 and nfrac <= NORM_MAX_FRAC, f"norm_out {nmax} ulp on {nfrac:.3e}"
        stats["norm_mismatch_frac"] = nfrac
    return stats
