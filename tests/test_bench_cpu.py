"""bench.py parts that need no GPU: the clock summary over timed windows, the
traffic table, the peaks fallback, and the reference arm (the CPU path on rank
0, the other ranks exiting without work)."""

import bench


def test_clock_summary_uses_only_samples_inside_windows():
    s = bench.ClockSampler(0)
    s.samples = [
        (1.0, 1965.0, 1965.0, 200.0, []),                 # idle, before the timed window
        (2.1, 1500.0, 1965.0, 980.0, ["sw_power_cap"]),
        (2.2, 1480.0, 1965.0, 990.0, ["sw_power_cap"]),
        (2.3, 1520.0, 1965.0, 985.0, []),
        (3.5, 1965.0, 1965.0, 300.0, []),                 # between windows
        (4.1, 1490.0, 1965.0, 975.0, ["sw_power_cap"]),
    ]
    out = s.summary([(2.0, 2.5), (4.0, 4.5)])
    assert out["samples"] == 4
    assert out["sm_mhz"] == 1495.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w"] == 982.5
    assert s.summary([(10.0, 11.0)])["samples"] == 0
    # a window shorter than the sampling period takes the samples just around it
    near = s.summary([(2.24, 2.26)], pad_s=0.1)
    assert near["samples"] == 2 and near["window_widened_s"] == 0.1
    assert s.summary([(2.24, 2.26)], pad_s=0.0)["samples"] == 0


def test_visible_devices_mapping(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench.ClockSampler(1).gpu == 5
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    assert bench.ClockSampler(2).gpu == 2


def test_traffic_table_and_peaks():
    assert bench.load_traffic("cfg4") > 0
    assert bench.load_traffic("no-such-workload") is None
    peaks, source = bench.load_peaks()
    assert peaks["bf16_tflops"] > 0 and source in ("measured", "fallback")


def _bench(args, rank):
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE="2")
    return subprocess.run([sys.executable, str(root / "bench.py"), *args], cwd=root, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_rank0_prints_one_line_other_ranks_exit_quietly():
    import json

    import time

    args = ["--impl", "reference", "--config", "cfg1", "--gpus", "2", "--steps", "1"]
    r1 = _bench(args, rank=1)
    assert r1.returncode == 0 and r1.stdout.strip() == "", r1.stderr[-2000:]
    t0 = time.perf_counter()
    r0 = _bench(args, rank=0)
    wall_ms = (time.perf_counter() - t0) * 1e3
    assert r0.returncode == 0, r0.stderr[-2000:]
    lines = [ln for ln in r0.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert line["warmup"] >= 3 and line["steps"] == 1 and line["n_gpus"] == 2
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == "cfg1"
    # The line reports the step it ran: its timed steps fit inside the process's wall time.
    assert line["ms_per_step"] * line["steps"] <= wall_ms
    assert line["workload_ms_extrapolated"] >= line["ms_per_step"]


def test_reference_arm_steps_fit_the_run_at_the_headline_size():
    """cfg4: one [8192 x 128] slice per step; 512 slices would take ~40 s per step,
    so a line that multiplied by the slice count would not fit the run."""
    import json
    import time

    t0 = time.perf_counter()
    r = _bench(["--impl", "reference", "--config", "cfg4", "--steps", "2", "--warmup", "3"], rank=0)
    wall_ms = (time.perf_counter() - t0) * 1e3
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["steps"] == 2 and line["ms_per_step"] * line["steps"] <= wall_ms
    assert line["workload_ms_extrapolated"] == line["ms_per_step"] * 512


def test_reference_arm_has_no_causal_mask():
    import json

    r = _bench(["--impl", "reference", "--config", "cfg1", "--causal"], rank=0)
    assert r.returncode == 0
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line
