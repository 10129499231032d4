"""GPU parity: the sm_100a kernel (through the public API and the C ABI)
against the CPU oracle and the reference's golden outputs."""
from pathlib import Path

import numpy as np
import pytest
import torch

from _compare import check_outputs, q_diff
from cases import CASES, case_inputs, stored_rows
from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant, launch_plan
from flagos_kernelgen_72h_shanghai_2026_b200.workloads import CONFIGS, Workload, make_inputs
from oracle.farq_oracle import fused_add_rmsnorm_group_quant_ref

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
MODES = {torch.int8: "int8", torch.float8_e4m3fn: "e4m3"}


def run_gpu(x, r, g, eps, G, q_dtype, dev, write_norm=True, ue8m0=False, norm_dtype=torch.bfloat16,
            rout_dtype=None, **kw):
    M, D = x.shape
    xd, rd, gd = x.to(dev), r.to(dev), g.to(dev)
    ro = torch.empty(M, D, dtype=rout_dtype or x.dtype, device=dev)
    no = torch.empty(M, D, dtype=norm_dtype, device=dev) if write_norm else None
    q = torch.empty(M, D, dtype=q_dtype, device=dev)
    s = torch.empty(M, D // G, dtype=torch.float32, device=dev)
    out = fused_add_rmsnorm_group_quant(xd, rd, gd, ro, no, q, s, eps, G, ue8m0=ue8m0, **kw)
    assert out[0] is ro and out[1] is no and out[2] is q and out[3] is s
    torch.cuda.synchronize(dev)
    return dict(residual_out=ro.cpu(), norm_out=None if no is None else no.cpu(),
                x_q=q.cpu(), x_scale=s.cpu())


def ref_dict(x, r, g, eps, G, mode, ue8m0=False, norm_dtype=torch.bfloat16, rout_dtype=None):
    ro, no, q, s = fused_add_rmsnorm_group_quant_ref(x, r, g, eps, G, mode, ue8m0,
                                                     residual_out_dtype=rout_dtype,
                                                     norm_out_dtype=norm_dtype)
    return dict(residual_out=ro, norm_out=no, x_q=q, x_scale=s)


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("name", list(CASES))
def test_int8_matches_reference_golden(cuda_dev, name):
    """q and scales from the reference's own kernels (run in Triton's
    interpreter) against the CUDA kernel; residual_out bit-exact (RNE)."""
    w, x, r, g = case_inputs(name)
    got = run_gpu(x, r, g, w.eps, w.group_size, torch.int8, cuda_dev)
    d = np.load(GOLDEN / f"{name}.npz")
    gs = torch.from_numpy(d["scale"])
    gq = torch.from_numpy(d["q"])
    assert ((stored_rows(name, got["x_scale"]) - gs).abs() / gs.abs()).max().item() <= 1e-6
    dq = q_diff(stored_rows(name, got["x_q"]), gq, "int8")
    assert int(dq.max()) <= 1 and (dq != 0).float().mean().item() <= 1e-3
    exp_ro = (x.float() + r.float()).to(x.dtype)
    assert torch.equal(got["residual_out"].view(torch.int16), exp_ro.view(torch.int16))
    # and the oracle, which pins norm_out too
    check_outputs(got, ref_dict(x, r, g, w.eps, w.group_size, "int8"), "int8")


# ---------------------------------------------------------------- configs
@pytest.mark.parametrize("cfg", [1, 2, 3, 4])
@pytest.mark.parametrize("q_dtype", [torch.float8_e4m3fn, torch.int8])
def test_benchmark_configs_vs_oracle(cuda_dev, cfg, q_dtype):
    w = CONFIGS[cfg]
    x, r, g = make_inputs(w)
    mode = MODES[q_dtype]
    got = run_gpu(x, r, g, w.eps, w.group_size, q_dtype, cuda_dev, ue8m0=w.ue8m0)
    check_outputs(got, ref_dict(x, r, g, w.eps, w.group_size, mode, w.ue8m0), mode, w.ue8m0)


def test_config5_sampled_rows(cuda_dev):
    """Full 262144 x 7168 call; rows are independent, so a spread of rows is
    checked against the oracle and residual_out is checked everywhere."""
    w = CONFIGS[5]
    x, r, g = make_inputs(w, device=cuda_dev)
    ro = torch.empty_like(x)
    q = torch.empty(w.M, w.D, dtype=w.q_dtype, device=cuda_dev)
    s = torch.empty(w.M, w.groups, dtype=torch.float32, device=cuda_dev)
    fused_add_rmsnorm_group_quant(x, r, g, ro, None, q, s, w.eps, w.group_size)
    for s0 in range(0, w.M, 32768):  # residual_out bit-exact, chunked fp32 temporaries
        e0 = s0 + 32768
        exp = (x[s0:e0].float() + r[s0:e0].float()).to(x.dtype)
        assert torch.equal(ro[s0:e0].view(torch.int16), exp.view(torch.int16))
    rows = torch.cat([torch.arange(0, 64), torch.randint(0, w.M, (448,),
                      generator=torch.Generator().manual_seed(1)), torch.arange(w.M - 64, w.M)])
    rows = rows.to(cuda_dev)
    got = dict(residual_out=ro[rows].cpu(), x_q=q[rows].cpu(), x_scale=s[rows].cpu())
    ref = ref_dict(x[rows].cpu(), r[rows].cpu(), g.cpu(), w.eps, w.group_size, "e4m3")
    check_outputs(got, ref, "e4m3")


# ---------------------------------------------------------------- shapes
SHAPES = [
    (1, 4096, 128), (2, 4096, 128), (127, 7168, 128), (129, 7168, 128), (3, 8192, 256),
    (300, 5120, 64), (17, 64, 8), (5, 256, 16), (9, 1024, 32), (33, 2048, 256),
    (64, 16384, 128), (1000, 6144, 128), (4, 12288, 64), (7, 13824, 128),
]


@pytest.mark.parametrize("M,D,G", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_shapes(cuda_dev, M, D, G, dtype):
    w = Workload("s", M, D, dtype=dtype, group_size=G, seed=M * 7 + D)
    x, r, g = make_inputs(w)
    for q_dtype in (torch.int8, torch.float8_e4m3fn):
        mode = MODES[q_dtype]
        got = run_gpu(x, r, g, w.eps, G, q_dtype, cuda_dev)
        check_outputs(got, ref_dict(x, r, g, w.eps, G, mode), mode)


@pytest.mark.parametrize("gamma_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("rout_dtype", [torch.float32, None])
@pytest.mark.parametrize("norm_dtype", [torch.float32, torch.float16])
def test_dtype_combinations(cuda_dev, gamma_dtype, rout_dtype, norm_dtype):
    w = Workload("d", 37, 3072, seed=11)
    x, r, g = make_inputs(w)
    g = g.to(gamma_dtype)
    got = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev, norm_dtype=norm_dtype,
                  rout_dtype=rout_dtype)
    ref = ref_dict(x, r, g, w.eps, 128, "e4m3", norm_dtype=norm_dtype, rout_dtype=rout_dtype)
    check_outputs(got, ref, "e4m3")


def test_zero_rows_and_huge_values(cuda_dev):
    w = Workload("z", 6, 4096, seed=3)
    x, r, g = make_inputs(w)
    x[1] = 0
    r[1] = 0
    x[3, :128] = 1.0e30  # r*gamma stays finite; sum(r*r) rounds to +inf in fp32
    r[3] = 0
    x[4, 5] = 1e4
    for q_dtype in (torch.int8, torch.float8_e4m3fn):
        mode = MODES[q_dtype]
        got = run_gpu(x, r, g, w.eps, 128, q_dtype, cuda_dev)
        ref = ref_dict(x, r, g, w.eps, 128, mode)
        assert torch.all(got["x_scale"][1] == torch.tensor(1e-12))
        assert torch.all(got["x_q"][1].view(torch.uint8) == 0)
        # row 3: sum(r*r) in fp64 is finite but rounds to +inf in fp32 -> inv_rms = 0,
        # every scale hits the 1e-12 floor and q is 0
        keep = [0, 1, 2, 4, 5]
        sub = {k: (v[keep] if v is not None else None) for k, v in got.items()}
        rsub = {k: v[keep] for k, v in ref.items()}
        check_outputs(sub, rsub, mode)
        assert torch.equal(got["x_q"][3].view(torch.uint8), ref["x_q"][3].view(torch.uint8))
        assert torch.equal(got["x_scale"][3], ref["x_scale"][3])


def test_norm_out_skipped_when_none_or_empty(cuda_dev):
    w = Workload("n", 50, 7168, seed=5)
    x, r, g = make_inputs(w)
    a = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev, write_norm=False)
    assert a["norm_out"] is None
    dev = cuda_dev
    empty = torch.empty(0, dtype=torch.bfloat16, device=dev)
    ro = torch.empty_like(x, device=dev)
    q = torch.empty(50, 7168, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty(50, 56, device=dev)
    out = fused_add_rmsnorm_group_quant(x.to(dev), r.to(dev), g.to(dev), ro, empty, q, s, w.eps, 128)
    assert out[1] is empty
    assert torch.equal(q.cpu().view(torch.uint8), a["x_q"].view(torch.uint8))


# ------------------------------------------------------- memory safety
def test_guard_padded_outputs_untouched(cuda_dev):
    """Outputs are row-strided windows inside canary-filled buffers: every
    byte outside the windows must survive (stand-in for a memory checker)."""
    dev = cuda_dev
    M, D, G = 77, 5120, 64
    w = Workload("g", M, D, group_size=G, seed=9)
    x, r, g = make_inputs(w)
    pad = 64  # elements of padding per row, half on each side, plus a row above and below
    bufs = []

    def canvas(dtype, cols):
        isz = torch.empty(0, dtype=dtype).element_size()
        raw = torch.full(((M + 2), (cols + pad) * isz), 0x5A, dtype=torch.uint8, device=dev)
        win = raw.view(dtype)[1:M + 1, pad // 2: pad // 2 + cols]
        bufs.append((raw, raw.clone(), (pad // 2) * isz, (pad // 2 + cols) * isz))
        return win

    ro = canvas(torch.bfloat16, D)
    no = canvas(torch.bfloat16, D)
    q = canvas(torch.float8_e4m3fn, D)
    s = canvas(torch.float32, D // G)
    fused_add_rmsnorm_group_quant(x.to(dev), r.to(dev), g.to(dev), ro, no, q, s, w.eps, G)
    torch.cuda.synchronize()
    for raw, before, c0, c1 in bufs:
        after = raw.clone()
        after[1:M + 1, c0:c1] = 0
        before[1:M + 1, c0:c1] = 0
        assert torch.equal(after, before), "a byte outside the output window changed"
    got = dict(residual_out=ro.cpu(), norm_out=no.cpu(), x_q=q.cpu(), x_scale=s.cpu())
    check_outputs(got, ref_dict(x, r, g, w.eps, G, "e4m3"), "e4m3")


def test_in_place_residual(cuda_dev):
    """residual_out may alias residual (or x), as in the reference (each
    element is read before it is written)."""
    w = Workload("i", 300, 7168, res_std=2.0, seed=13)
    x, r, g = make_inputs(w)
    ref = ref_dict(x, r, g, w.eps, 128, "e4m3")
    for alias in ("residual", "x"):
        xd, rd, gd = x.cuda(), r.cuda(), g.cuda()
        ro = rd if alias == "residual" else xd
        q = torch.empty(300, 7168, dtype=torch.float8_e4m3fn, device="cuda")
        s = torch.empty(300, 56, device="cuda")
        no = torch.empty(300, 7168, dtype=torch.bfloat16, device="cuda")
        fused_add_rmsnorm_group_quant(xd, rd, gd, ro, no, q, s, w.eps, 128)
        torch.cuda.synchronize()
        got = dict(residual_out=ro.cpu(), norm_out=no.cpu(), x_q=q.cpu(), x_scale=s.cpu())
        check_outputs(got, ref, "e4m3")


def test_row_strided_inputs(cuda_dev):
    w = Workload("st", 40, 4096, seed=17)
    x, r, g = make_inputs(w)
    big_x = torch.zeros(40, 4096 + 256, dtype=torch.bfloat16, device="cuda")
    big_r = torch.zeros(40, 4096 + 512, dtype=torch.bfloat16, device="cuda")
    big_x[:, 128:128 + 4096] = x.cuda()
    big_r[:, :4096] = r.cuda()
    xv, rv = big_x[:, 128:128 + 4096], big_r[:, :4096]
    ro = torch.empty(40, 4096, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(40, 4096, dtype=torch.int8, device="cuda")
    s = torch.empty(40, 32, device="cuda")
    fused_add_rmsnorm_group_quant(xv, rv, g.cuda(), ro, None, q, s, w.eps, 128)
    torch.cuda.synchronize()
    got = dict(residual_out=ro.cpu(), x_q=q.cpu(), x_scale=s.cpu())
    check_outputs(got, ref_dict(x, r, g, w.eps, 128, "int8"), "int8")


# ------------------------------------------------------------ plumbing
def test_tuning_knobs_do_not_change_results(cuda_dev):
    w = Workload("t", 1000, 7168, seed=19)
    x, r, g = make_inputs(w)
    base = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev)
    for ctas, teams, stages, k in ((1, 1, 1, 0), (1, 4, 2, 0), (2, 1, 1, 0), (1, 2, 3, 0),
                                   (1, 0, 0, 4), (1, 0, 0, 8), (2, 2, 1, 2), (1, 3, 2, 5)):
        got = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev,
                      _tune_ctas_per_sm=ctas, _tune_teams_per_cta=teams, _tune_stages=stages,
                      _tune_vec_per_thread=k)
        for key in base:
            if base[key] is not None:
                assert torch.equal(got[key].view(torch.uint8), base[key].view(torch.uint8)), \
                    (ctas, teams, stages, k, key)


def test_side_stream_and_cuda_graph(cuda_dev):
    w = Workload("cg", 512, 7168, seed=23)
    x, r, g = make_inputs(w)
    xd, rd, gd = x.cuda(), r.cuda(), g.cuda()
    ro = torch.empty_like(xd)
    q = torch.empty(512, 7168, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(512, 56, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        fused_add_rmsnorm_group_quant(xd, rd, gd, ro, None, q, s, w.eps, 128)
    st.synchronize()
    first = (ro.clone(), q.clone(), s.clone())
    ro.zero_(); q.view(torch.uint8).zero_(); s.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        fused_add_rmsnorm_group_quant(xd, rd, gd, ro, None, q, s, w.eps, 128)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(ro, first[0]) and torch.equal(q.view(torch.uint8), first[1].view(torch.uint8))
    assert torch.equal(s, first[2])


def test_status_word_stays_zero(cuda_dev):
    w = Workload("sw", 2000, 7168, seed=29)
    x, r, g = make_inputs(w, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ro = torch.empty_like(x)
    q = torch.empty(2000, 7168, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(2000, 56, device="cuda")
    for _ in range(3):
        fused_add_rmsnorm_group_quant(x, r, g, ro, None, q, s, w.eps, 128, _status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_bounded_wait_times_out_into_status_word(cuda_dev):
    """A device wait that nothing satisfies (test-only flag, 1 ms limit)
    returns through the status word; the context stays usable."""
    w = Workload("to", 1184, 4096, seed=31)
    x, r, g = make_inputs(w, device="cuda")
    ro = torch.empty_like(x)
    q = torch.empty(w.M, w.D, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(w.M, w.groups, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    fused_add_rmsnorm_group_quant(x, r, g, ro, None, q, s, w.eps, 128, _status=status,
                                  _test_force_timeout=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 9  # FARQ_ERR_DEVICE_TIMEOUT
    status.zero_()
    fused_add_rmsnorm_group_quant(x, r, g, ro, None, q, s, w.eps, 128, _status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = dict(residual_out=ro.cpu(), x_q=q.cpu(), x_scale=s.cpu())
    check_outputs(got, ref_dict(x.cpu(), r.cpu(), g.cpu(), w.eps, 128, "e4m3"), "e4m3")


@pytest.mark.parametrize("chunk", [64, 500, 4096])
def test_host_buffer_entry_matches_device_entry(cuda_dev, chunk):
    from flagos_kernelgen_72h_shanghai_2026_b200 import fused_add_rmsnorm_group_quant_host
    w = Workload("h", 1300, 7168, res_std=2.0, seed=37)
    x, r, g = make_inputs(w)
    dev = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev)
    hx, hr = x.pin_memory(), r.pin_memory()
    ro = torch.empty_like(hx).pin_memory()
    no = torch.empty(w.M, w.D, dtype=torch.bfloat16).pin_memory()
    q = torch.empty(w.M, w.D, dtype=torch.float8_e4m3fn).pin_memory()
    s = torch.empty(w.M, w.groups).pin_memory()
    for _ in range(2):  # second call reuses the cached staging pipeline
        out = fused_add_rmsnorm_group_quant_host(hx, hr, g, ro, no, q, s, w.eps, 128,
                                                 device=cuda_dev, chunk_rows=chunk)
        torch.cuda.current_stream().synchronize()
        assert out[0] is ro and out[2] is q
        got = dict(residual_out=ro, norm_out=no, x_q=q, x_scale=s)
        for k in got:
            assert torch.equal(got[k].view(torch.uint8), dev[k].view(torch.uint8)), k
        ro.zero_(); q.view(torch.uint8).zero_(); s.zero_()


def test_column_major_scales(cuda_dev):
    """x_scale as a transposed [groups, ld] buffer (the layout blockwise-FP8
    GEMMs read); every other output identical to the row-major call."""
    w = Workload("cm", 300, 7168, seed=41)
    x, r, g = make_inputs(w)
    base = run_gpu(x, r, g, w.eps, 128, torch.float8_e4m3fn, cuda_dev)
    ld = 304  # M rounded up to a multiple of 16
    buf = torch.full((w.groups, ld), -1.0, device="cuda")
    s_cm = buf[:, :w.M].t()
    ro = torch.empty(w.M, w.D, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(w.M, w.D, dtype=torch.float8_e4m3fn, device="cuda")
    fused_add_rmsnorm_group_quant(x.cuda(), r.cuda(), g.cuda(), ro, None, q, s_cm, w.eps, 128)
    torch.cuda.synchronize()
    assert torch.equal(s_cm.cpu(), base["x_scale"])
    assert torch.all(buf[:, w.M:] == -1.0)  # padding columns untouched
    assert torch.equal(q.cpu().view(torch.uint8), base["x_q"].view(torch.uint8))


def test_errors_raise(cuda_dev):
    dev = cuda_dev
    x = torch.zeros(4, 1000, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        fused_add_rmsnorm_group_quant(x, x, torch.ones(1000, dtype=torch.bfloat16, device=dev),
                                      x.clone(), None, torch.empty(4, 1000, dtype=torch.int8, device=dev),
                                      torch.empty(4, 10, device=dev), 1e-6, 100)
    x = torch.zeros(4, 1024, dtype=torch.float32, device=dev)
    with pytest.raises(TypeError):
        fused_add_rmsnorm_group_quant(x, x, torch.ones(1024, device=dev), x.clone(), None,
                                      torch.empty(4, 1024, dtype=torch.int8, device=dev),
                                      torch.empty(4, 8, device=dev), 1e-6, 128)
    xb = torch.zeros(4, 1024, dtype=torch.bfloat16, device=dev)
    xm = torch.zeros(4 * 1024 + 4, dtype=torch.bfloat16, device=dev)[4:].view(4, 1024)  # 8-byte offset
    with pytest.raises(ValueError, match="misaligned"):
        fused_add_rmsnorm_group_quant(xm, xb, torch.ones(1024, dtype=torch.bfloat16, device=dev),
                                      xb.clone(), None, torch.empty(4, 1024, dtype=torch.int8, device=dev),
                                      torch.empty(4, 8, device=dev), 1e-6, 128)


def test_launch_plan_reports_persistent_grid(cuda_dev):
    p = launch_plan(4096, 7168)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert p["team_threads"] * p["vec_per_thread"] * 8 >= 7168
    assert p["grid"] == sms and p["teams"] >= 1 and p["stages"] >= 1
    small = launch_plan(5, 7168)
    assert small["grid"] == 5 and small["teams"] == 1
    assert small["team_threads"] == 448 and small["vec_per_thread"] == 2  # widest team
