"""bench.py's reference arm keeps the JSON line contract (CPU only: the arm is PyTorch CPU)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "3", "--warmup", "3"], capture_output=True, text=True,
                       timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-500:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] in ("port", "reference")
    assert "workload" in d["config"]


def test_bench_rejects_fewer_than_three_warmup_steps_by_raising_them():
    src = (ROOT / "bench.py").read_text()
    assert "args.warmup = max(args.warmup, 3)" in src


def test_clock_summary_reads_the_sampled_fields():
    """The clock sampler's summary (no GPU: lines as nvidia-smi prints them with nounits)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    s = bench.ClockSampler(0)
    s.lines = [(10.0, "0, 1680, 1965, 702.5, 0x4, Not Active, Not Active, Not Active, Active"),
               (10.2, "0, 1700, 1965, 710.1, 0x4, Not Active, Not Active, Not Active, Active"),
               (10.4, "0, 1690, 1965, 706.0, 0x4, Not Active, Not Active, Not Active, Active"),
               (99.0, "0, 120, 1965, 199.0, 0x1, Not Active, Not Active, Not Active, Not Active")]
    out = s.summary(10.1, 10.3)
    assert out["samples"] == 3 and out["sm_mhz"] == 1690.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["power_w"] == 706.0
