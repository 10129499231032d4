"""The CPU oracle against the reference's own outputs (golden fixtures made by
running src/task01_fused_add_rmsnorm_group_quant.py under TRITON_INTERPRET=1)
and against known properties of the e4m3 / UE8M0 encodings."""
import numpy as np
import pytest
import torch

from _compare import Q_MAX_FRAC, SCALE_RTOL, q_diff
from cases import CASES, case_inputs, input_digest
from oracle.farq_oracle import (e4m3_bytes, e4m3_rne_sat, fused_add_rmsnorm_group_quant_ref,
                                pow2_ceil)
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference_golden(name):
    w, x, r, g = case_inputs(name)
    d = np.load(GOLDEN / f"{name}.npz")
    assert str(d["digest"]) == input_digest(x, r, g), "seeded inputs drifted from the fixture"
    ro, no, q, s = fused_add_rmsnorm_group_quant_ref(x, r, g, w.eps, w.group_size, "int8")
    gq = torch.from_numpy(d["q"])
    gs = torch.from_numpy(d["scale"])
    rel = ((s - gs).abs() / gs.abs()).max().item()
    assert rel <= SCALE_RTOL
    dq = q_diff(q, gq, "int8")
    assert int(dq.max()) <= 1
    assert (dq != 0).float().mean().item() <= Q_MAX_FRAC


def test_zero_row_hits_scale_floor():
    w, x, r, g = case_inputs("full_row_5x8192_g256_zero_row")
    _, _, q, s = fused_add_rmsnorm_group_quant_ref(x, r, g, w.eps, w.group_size, "int8")
    assert torch.all(s[2] == torch.tensor(1e-12, dtype=torch.float32))
    assert torch.all(q[2] == 0)


def test_int8_is_truncation_not_round():
    # bf16(1.1) = 1.1015625; with group max 4.0, v = 1.1015625/4*127 = 34.97 -> 34 (trunc), not 35
    x = torch.tensor([[4.0, 1.1, -1.1] + [0.0] * 5], dtype=torch.bfloat16)
    r = torch.zeros_like(x)
    g = torch.ones(8, dtype=torch.bfloat16)
    _, _, q, s = fused_add_rmsnorm_group_quant_ref(x, r, g, 1e-6, 8, "int8")
    assert int(q[0, 1]) == 34 and int(q[0, 2]) == -34
    assert int(q[0, 0]) in (126, 127)  # the group maximum sits on 127 up to rounding


def test_e4m3_encoder_matches_torch_cast_in_range():
    g = torch.Generator().manual_seed(0)
    v = torch.randn(200000, generator=g) * torch.exp2(torch.randint(-12, 9, (200000,), generator=g).float())
    v = v.clamp(-448, 448)
    ours = e4m3_bytes(e4m3_rne_sat(v))
    theirs = v.to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(ours, theirs)


def test_e4m3_encoder_grid_midpoints_and_saturation():
    grid = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    fin = grid[torch.isfinite(grid)]
    # every grid value maps to itself
    assert torch.equal(e4m3_rne_sat(fin), fin)
    pos = torch.unique(fin[fin >= 0])
    mids = (pos[:-1] + pos[1:]) / 2
    out = e4m3_rne_sat(mids)
    lo_codes = pos[:-1].to(torch.float8_e4m3fn).view(torch.uint8)
    hi_codes = pos[1:].to(torch.float8_e4m3fn).view(torch.uint8)
    even = torch.where(lo_codes % 2 == 0, pos[:-1], pos[1:])
    assert torch.equal(out, even)
    sat = e4m3_rne_sat(torch.tensor([449.0, 464.0, 500.0, 1e30, float("inf"), -1e9]))
    assert sat.tolist() == [448.0, 448.0, 448.0, 448.0, 448.0, -448.0]
    assert torch.isnan(e4m3_rne_sat(torch.tensor([float("nan")]))).all()
    del hi_codes


def test_pow2_ceil():
    s = torch.tensor([1.0, 1.5, 0.75, 3.0e-12, 2.0 ** -20, 1.0000001, 448.0])
    out = pow2_ceil(s)
    assert out.tolist() == [1.0, 2.0, 1.0, 2.0 ** -38, 2.0 ** -20, 2.0, 512.0]


def test_e4m3_mode_saturates_and_round_trips():
    w, x, r, g = case_inputs("segmented_160x7168_outliers")
    ro, no, q, s = fused_add_rmsnorm_group_quant_ref(x, r, g, w.eps, w.group_size, "e4m3")
    deq = q.view(torch.float8_e4m3fn).float().view(w.M, w.groups, w.group_size) * s[:, :, None]
    norm = no.float().view(w.M, w.groups, w.group_size)
    # group maximum maps to +-448 (within one e4m3 step), dequantised error
    # is at most half an e4m3 ulp of the value (2^-4 relative) plus bf16 rounding of norm
    assert q.view(torch.float8_e4m3fn).float().abs().amax().item() == 448.0
    err = (deq - norm).abs()
    assert bool((err <= norm.abs() * 0.0625 + s[:, :, None] * 2 ** -9 + norm.abs() * 2 ** -8).all())
