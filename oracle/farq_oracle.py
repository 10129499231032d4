"""CPU oracle for fused residual-add + RMSNorm + per-token group quantisation.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path; it is
imported only by tests/ and __graft_entry__.smoke(). (The timed CPU baseline
is the plain-C restatement in farq_oracle.c, which matches this module bit
for bit.) The
product path (flagos_kernelgen_72h_shanghai_2026_b200) never calls it.

It restates, in vectorised fp32 torch-on-CPU code, the per-row arithmetic of
sinpeyw/flagos-kernelgen-72h-shanghai-2026
src/task01_fused_add_rmsnorm_group_quant.py:
  r        = f32(x) + f32(residual)                     :1151-1157 (:84-85)
  residual_out = r cast to the output dtype (RNE)        :1160 (:87)
  inv_rms  = rsqrt(sum(r*r) / D + eps)                   :1274-1278 (:86, :97)
  w        = r * f32(gamma)                              :1163-1164 (:89-90)
  gmax[g]  = max |w| over the group                      :1165-1167 (:91-95)
  norm     = w * inv_rms                                 :1089 (:98)
  scale    = max(gmax * (inv_rms / 127), 1e-12)          :1090 (:99)
  q        = trunc(clamp(norm * (1/scale), -127, 127))   :1091-1104 (:100-116)
The cast to int is truncation toward zero (Triton's fp->int `.to`), which a
run of the reference kernels under TRITON_INTERPRET=1 confirms (the golden
fixtures in tests/golden/ were produced that way).

Precision choices, identical in the CUDA kernel:
  * sum(r*r) is accumulated in float64 and rounded to fp32 once, here and
    in the kernel, so inv_rms is independent of the summation order. (The
    reference accumulates in fp32 in Triton's tree order; its inv_rms can
    differ by an ulp, which flips a group's maximum element between 126 and
    127 — that is where the residual q mismatches against the golden
    fixtures come from.)
  * inv_rms = 1 / sqrt(mean + eps) with IEEE fp32 sqrt and division (the
    reference's Triton rsqrt is an approximation; both stay within the
    stated tolerances).
  * 1/scale is an IEEE fp32 reciprocal.

Extensions with no reference code (pinned only by this restatement):
  * E4M3 mode: scale = max(gmax * (inv_rms / 448), 1e-12);
    q = round-to-nearest-even of norm*(1/scale) onto the e4m3fn grid,
    saturating at ±448 (e4m3_rne_sat below).
  * UE8M0: scale rounded up to a power of two from its fp32 bits.

Parity for int8 mode is pinned against the reference's own kernels run in
Triton's interpreter (tests/golden/); e4m3/UE8M0 parity is unpinned by the
reference, which has no such mode.
"""
from __future__ import annotations

import numpy as np
import torch

QMAX_INT8 = 127.0
QMAX_E4M3 = 448.0
SCALE_FLOOR = 1.0e-12


def e4m3_rne_sat(v: torch.Tensor) -> torch.Tensor:
    """fp32 -> fp32 values on the float8_e4m3fn grid: round to nearest even,
    saturate finite values to ±448. NaN stays NaN.

    e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; normal exponents
    -6..8; subnormal spacing 2^-9; largest finite 448 = 1.75 * 2^8.
    Rounding is done as rint(|v| / q) * q with q the grid spacing at |v|'s
    binade (an exact power-of-two scaling), rint being round-half-even.
    """
    v = v.float()
    a = v.abs()
    # binade exponent, clamped to the normal range floor (-6) for subnormals
    _, e = torch.frexp(a)                      # a = m * 2^e, m in [0.5, 1)
    e = (e - 1).clamp(min=-6)
    q = torch.ldexp(torch.ones_like(a), (e - 3).to(torch.int32))
    r = torch.round(a / q) * q                  # torch.round is half-to-even
    r = torch.minimum(r, torch.full_like(r, QMAX_E4M3))
    r = torch.where(torch.isnan(v), v, r)
    return torch.copysign(r, v)


def e4m3_bytes(v: torch.Tensor) -> torch.Tensor:
    """float8_e4m3fn bit patterns (uint8) of fp32 values already on the grid."""
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def pow2_ceil(s: torch.Tensor) -> torch.Tensor:
    """Round positive normal fp32 values up to a power of two, from the bits."""
    b = s.float().contiguous().view(torch.int32)
    mant = b & 0x007FFFFF
    up = (b & ~0x007FFFFF) + 0x00800000
    return torch.where(mant != 0, up, b).view(torch.float32)


def fused_add_rmsnorm_group_quant_ref(x: torch.Tensor, residual: torch.Tensor,
                                      gamma: torch.Tensor, eps: float, group_size: int,
                                      q_mode: str = "int8", ue8m0: bool = False,
                                      residual_out_dtype: torch.dtype | None = None,
                                      norm_out_dtype: torch.dtype = torch.bfloat16):
    """Returns (residual_out, norm_out, q, scale) on CPU.

    q is int8 for q_mode="int8" and the uint8 bit patterns of float8_e4m3fn
    for q_mode="e4m3". norm_out is in ``norm_out_dtype``.
    """
    x = x.detach().cpu()
    residual = residual.detach().cpu()
    gamma = gamma.detach().cpu()
    M, D = x.shape
    G = int(group_size)
    assert D % G == 0
    residual_out_dtype = residual_out_dtype or x.dtype
    r = x.float() + residual.float()
    residual_out = r.to(residual_out_dtype)
    ss = (r.double() * r.double()).sum(dim=1).float()
    mean = ss / torch.tensor(float(D), dtype=torch.float32)
    # numpy's float32 sqrt is the correctly rounded IEEE one; torch's CPU
    # sqrt is not (it is off by an ulp on ~0.6% of inputs)
    inv = 1.0 / torch.from_numpy(np.sqrt((mean + torch.tensor(eps, dtype=torch.float32)).numpy()))
    w = r * gamma.float()[None, :]
    gmax = w.abs().view(M, D // G, G).amax(dim=2)
    norm = w * inv[:, None]
    qmax = QMAX_INT8 if q_mode == "int8" else QMAX_E4M3
    step = inv / torch.tensor(qmax, dtype=torch.float32)
    scale = torch.clamp(gmax * step[:, None], min=SCALE_FLOOR)
    if ue8m0:
        scale = pow2_ceil(scale)
    isc = 1.0 / scale
    v = (norm.view(M, D // G, G) * isc[:, :, None]).view(M, D)
    if q_mode == "int8":
        q = torch.clamp(v, -QMAX_INT8, QMAX_INT8).trunc().to(torch.int8)
    elif q_mode == "e4m3":
        q = e4m3_bytes(e4m3_rne_sat(v))
    else:
        raise ValueError(f"q_mode {q_mode!r}")
    return residual_out, norm.to(norm_out_dtype), q, scale
