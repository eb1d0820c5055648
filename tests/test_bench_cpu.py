"""bench.py helpers that need no GPU: the clock summary over timed windows,
the traffic table and the peaks fallback."""

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
