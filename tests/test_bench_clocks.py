"""The benchmark's clock summary keeps only nvidia-smi samples taken inside
the timed region (or the nearest ones when the region is shorter than the
sampling interval) and reports the throttle reasons seen there."""
import datetime
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _line(t: float, mhz: int, cap: str = "Not Active", thermal: str = "Not Active") -> str:
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"0, {mhz}, 1965, 700.00 W, 0x0, Not Active, Not Active, {thermal}, {cap}, {ts}\n"


def _sampler(lines):
    fd, path = tempfile.mkstemp(suffix=".csv")
    with os.fdopen(fd, "w") as f:
        f.writelines(lines)
    s = bench.ClockSampler(0)
    s.path = path
    return s


def test_samples_inside_window_only():
    t0 = 1_700_000_000.0
    lines = [_line(t0 - 2, 900, thermal="Active")] + [_line(t0 + 0.05 * i, 1900 + i, cap="Active") for i in range(5)]
    s = _sampler(lines)
    s.mark(t0, t0 + 0.25)
    out = s.summary()
    assert out["samples"] == 5 and out["sampled"] == "timed region"
    assert out["sm_mhz"] == 1902 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]  # the thermal sample was before the window


def test_short_window_uses_nearest_samples():
    t0 = 1_700_000_000.0
    lines = [_line(t0 + 0.1 * i, 1800 + 10 * i) for i in range(10)]
    s = _sampler(lines)
    s.mark(t0 + 0.42, t0 + 0.44)  # no sample inside
    out = s.summary()
    assert out["samples"] == 3 and out["sampled"].startswith("3 samples nearest")
    assert out["sm_mhz"] == 1840 and out["reasons"] == []
