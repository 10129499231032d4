"""The CPU oracle against the reference's own outputs (golden fixtures made by
running src/task01_fused_add_rmsnorm_group_quant.py under TRITON_INTERPRET=1)
and against known properties of the e4m3 / UE8M0 encodings."""
import numpy as np
import pytest
import torch

from _compare import Q_MAX_FRAC, SCALE_RTOL, q_diff
from cases import CASES, case_inputs, input_digest, stored_rows
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
    q, s = stored_rows(name, q), stored_rows(name, s)
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
    even = torch.where(lo_codes % 2 == 0, pos[:-1], pos[1:])
    assert torch.equal(out, even)
    sat = e4m3_rne_sat(torch.tensor([449.0, 464.0, 500.0, 1e30, float("inf"), -1e9]))
    assert sat.tolist() == [448.0, 448.0, 448.0, 448.0, 448.0, -448.0]
    assert torch.isnan(e4m3_rne_sat(torch.tensor([float("nan")]))).all()


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


@pytest.mark.parametrize("cfg", ["bf16_g128", "fp16_g64_ue8m0", "outliers", "zero_row", "small_g"])
@pytest.mark.parametrize("mode", ["int8", "e4m3"])
def test_c_oracle_matches_torch_oracle_bit_for_bit(cfg, mode):
    """Two independent CPU restatements (torch and plain C) agree exactly."""
    from oracle.c_oracle import fused_add_rmsnorm_group_quant_c
    from flagos_kernelgen_72h_shanghai_2026_b200.workloads import Workload, make_inputs
    ue8m0 = False
    if cfg == "bf16_g128":
        w = Workload("c1", 64, 7168, res_std=2.0, seed=61)
    elif cfg == "fp16_g64_ue8m0":
        w = Workload("c2", 48, 5120, dtype=torch.float16, group_size=64, eps=1e-5, seed=62)
        ue8m0 = True
    elif cfg == "outliers":
        w = Workload("c3", 100, 7168, outlier_channels=8, outlier_row_frac=0.05, seed=63)
    elif cfg == "zero_row":
        w = Workload("c4", 5, 8192, group_size=256, seed=64)
    else:
        w = Workload("c5", 33, 1024, group_size=8, seed=65)
    x, r, g = make_inputs(w)
    if cfg == "zero_row":
        x[2] = 0
        r[2] = 0
    ref = fused_add_rmsnorm_group_quant_ref(x, r, g, w.eps, w.group_size, mode, ue8m0)
    got = fused_add_rmsnorm_group_quant_c(x, r, g, w.eps, w.group_size, mode, ue8m0, threads=4)
    names = ("residual_out", "norm_out", "q", "scale")
    for name, a, b in zip(names, got, ref):
        assert torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)), name
