"""bench.py's reference arm runs on the CPU alone: one JSON line with the
contract's keys (impl, metric, value, unit, cpu_baseline with kind / cores /
sample, e2e with zero copy bytes) and the reference's own CPU numbers beside
it.  Also the argument check on --warmup."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 3 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    if d.get("reference_q8_0_config1"):
        assert d["reference_q8_0_config1"]["kind"] == "reference"
        assert d["reference_q8_0_config1"]["value_1_thread"] > 0
    if d.get("reference_expert_chunk_q8_0_config5"):
        assert d["reference_expert_chunk_q8_0_config5"]["s_per_window"] > 0


def test_warmup_below_three_is_refused():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--warmup", "2"],
                       cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode != 0 and "warmup" in r.stderr


def test_clock_summary_keeps_the_load_window():
    """Samples outside the marked replay window (idle clocks before and
    after it) are left out, and so are idle samples inside it; without a
    window, every sample under load counts."""
    import time
    import bench
    c = bench.ClockSampler("00000000:e5:00.0")
    t = time.time()
    c.lines = [(t + 0.1 * i, f"00000000:E5:00.0, {1965 if 10 <= i < 30 else 600}, 1965, 700, "
                f"{90 if 10 <= i < 30 else 0}, Not Active, Not Active, Not Active, "
                f"{'Active' if i == 35 else 'Not Active'}") for i in range(40)]
    s = c.summary()
    assert s["samples"] == 20 and s["sm_mhz"] == 1965.0 and s["reasons"] == []
    c.window = (t + 1.0, t + 3.0)
    s = c.summary()
    assert s["samples_all"] == 19 and s["samples"] == 18  # the idle sample at the end is left out
    assert s["sm_mhz"] == 1965.0 and s["reasons"] == []
    assert s["gpu"] == "00000000:e5:00.0" and "replays" in s["window"]
