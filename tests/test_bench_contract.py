"""bench.py prints one JSON line with the keys the benchmark driver reads.

CPU: the reference arm (the reference library compiled from its sources) on a
small workload.  GPU: our arm on a small workload with every required key,
the roofline block, the CPU baseline, the end-to-end number and the clocks."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config"}


def run_bench(*args, timeout=600):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO,
                         capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    if not os.path.exists(os.path.join(REPO, "oracle", "_ref")):
        pytest.skip("oracle/_ref not built")
    line = run_bench("--impl", "reference", "--workload", "square512", "--steps", "1", "--warmup", "3")
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    assert BASE_KEYS <= set(line), BASE_KEYS - set(line)
    assert line["impl"] == "reference" and line["value"] > 0 and line["warmup"] >= 3
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"] == "square512"


@pytest.mark.gpu
def test_our_arm_line():
    line = run_bench("--workload", "square4096", "--steps", "3", "--warmup", "3", "--head-only")
    assert BASE_KEYS <= set(line), BASE_KEYS - set(line)
    assert line["n_gpus"] == 1 and line["value"] > 0 and line["higher_is_better"] is True
    r = line["roofline"]
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(r)
    assert 0 < r["frac"] < 1.5 and abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-9
    assert line["cpu_baseline"]["value"] > 0 and line["cpu_baseline"]["kind"] == "reference"
    e2e = line["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    assert line["gpu_launches"] >= line["steps"]
    assert "sm_mhz" in line["clocks"] and "reasons" in line["clocks"]


def test_clock_window_keeps_only_timed_samples():
    """The clock record counts only samples inside the timed region; a region
    shorter than one sampling interval takes the first sample after its start."""
    sys.path.insert(0, REPO)
    import bench
    cs = bench.ClockSampler(0)
    cs.samples = [(0.0, 1965, 1965, 200.0, set()), (1.0, 1400, 1965, 990.0, {"sw_power_cap"}),
                  (2.0, 1300, 1965, 995.0, {"sw_power_cap"}), (3.0, 1965, 1965, 210.0, set())]
    cs.t0, cs.t1 = 0.5, 2.5
    s = cs.summary(1965.0)
    assert s["samples"] == 2 and s["sm_mhz"] == 1350 and s["reasons"] == ["sw_power_cap"]
    assert s["power_w_max"] == 995.0
    cs.t0, cs.t1 = 2.2, 2.3
    s = cs.summary(1965.0)
    assert s["samples"] == 1 and s["sm_mhz"] == 1965 and s["reasons"] == []


@pytest.mark.gpu
def test_default_workload_sub_records():
    """The default (batched) line carries an end-to-end number for every mode,
    the 8192^3 record (TF32 with its own clock record) and the sustained run."""
    line = run_bench("--steps", "3", "--warmup", "3", "--no-cpu-baseline")
    assert line["config"]["workload"] == "batched" and line["config"]["global_batch"] == 64
    for mode in ("tf32", "3xtf32", "exact"):
        e2e = line["modes"][mode]["e2e"]
        assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] == 2 * 64 * 2048 * 2048 * 4
        assert e2e["d2h_bytes_per_step"] == 64 * 2048 * 2048 * 4
    sq = line["square8192"]
    for mode in ("tf32", "3xtf32", "exact"):
        assert sq[mode]["tflops"] > 0 and sq[mode]["launches_per_step"] >= 1
    assert "sm_mhz" in sq["tf32"]["clocks"]
    sus = line["sustained"]
    assert sus["seconds"] >= 1.0 and sus["tflops_per_gpu"] > 0 and "reasons" in sus["clocks"]
