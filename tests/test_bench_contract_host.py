"""The reference arm of bench.py on the host (no GPU): one JSON line with the
contract's keys, the CPU restatement's own numbers in cpu_baseline and e2e,
and at least three warm-up steps whatever was asked."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3
    assert d["higher_is_better"] is True and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert "sample" in cb
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    """Under torchrun only rank 0 runs and prints the reference line; the
    other ranks return 0 at once, printing nothing."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "3"], capture_output=True,
                       text=True, timeout=300, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def _bench():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_work_per_unit():
    """The roofline numerators: the causal prefill FLOPs of one step and the
    decode step's HBM bytes, 196,608·L + 393,216 at B = 64, H = 12, summing to
    27,443,331,072 over the 128 steps L = 1025 … 1152."""
    b = _bench()
    assert b.FLOPS_PER_STEP == 68_753_031_168
    assert b.dec_bytes(1) == 196_608 + 393_216
    assert sum(b.dec_bytes(L) for L in range(1025, 1153)) == 27_443_331_072


def test_peaks_and_traffic_are_read_from_committed_files():
    b = _bench()
    p = b.load_peaks()
    assert p["hbm_gbs"] > 0 and p["bf16_tflops"] > 0
    assert p["source"] == ("measured" if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json"))
                           else "fallback")
    names = [f[:-3] for f in os.listdir(os.path.join(ROOT, "profiles")) if f.endswith(".md")]
    with_traffic = [n for n in names if b.load_traffic(n) is not None]
    assert with_traffic and all(b.load_traffic(n) > 0 for n in with_traffic)
    assert b.load_traffic("no_such_profile") is None


def test_clock_samples_summary():
    """Median SM clock and the throttle reasons seen Active (nvidia-smi's CSV
    without units)."""
    b = _bench()
    lines = ["0, 1800, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
             "0, 1900, 1965, 900.3, 0x4, Not Active, Not Active, Not Active, Active",
             "0, 1700, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active",
             "garbage"]
    s = b.ClockSampler.summarise(lines)
    assert s == {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                 "samples": 3}
