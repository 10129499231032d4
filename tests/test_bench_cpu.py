"""bench.py's reference arm (CPU only) keeps the JSON-line contract."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "3", "--warmup", "3", "--ref-budget", "2"],
                         capture_output=True, text=True, timeout=300, check=True).stdout
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "cfg5_sharded_262144x7168"
    assert d["scaling"] == "strong" and d["dtype"] == "fp32"
    assert d["rows_per_step"] >= 16


def test_both_arms_share_one_config():
    """The repo arm and the reference arm build `config` with the same
    function, so a driver can pair their lines at every N."""
    sys.path.insert(0, str(ROOT))
    import bench
    from flagos_kernelgen_72h_shanghai_2026_b200.workloads import CONFIGS
    for n in (1, 2, 8):
        c = bench.line_config(CONFIGS[5], n, "strong")
        assert c["M"] == 262144 and c["M_per_gpu"] == 262144 // n
        assert c["bytes_per_call"] == 262144 * 7168 * 7 + 262144 * 56 * 4 + n * 2 * 7168


def test_warmup_below_three_is_refused():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "3", "--warmup", "2"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode != 0 and "warmup" in r.stderr
