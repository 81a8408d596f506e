"""``ClockSampler.summary`` (the ``clocks`` field of ``bench.py``'s line) on
synthetic nvidia-smi CSV: the median SM clock is taken over samples under
load (power above 200 W), the throttle reasons are those active under load,
the max clock over all samples, and unreadable lines are skipped."""

import os
import tempfile

from nano_megatron_b200.utils.timing import ClockSampler


def _summary(lines):
    fd, path = tempfile.mkstemp(suffix=".csv")
    with os.fdopen(fd, "w") as f:
        f.write("\n".join(lines) + "\n")
    s = ClockSampler()
    s.path = path
    out = s.summary()
    assert not os.path.exists(path)  # the sample file is removed
    return out


def _row(sm, power, active="Not Active", hw="Not Active", thermal="Not Active", sw_thermal="Not Active",
         cap="Not Active"):
    return f"0, {sm}, 1965, {power}, {active}, {hw}, {thermal}, {sw_thermal}, {cap}"


def test_median_under_load_and_reasons():
    lines = [_row(1965, 120.0), _row(1965, 150.0)]  # idle before the timed region
    lines += [_row(mhz, 990.0, cap="Active") for mhz in (1400, 1425, 1410, 1440, 1395)]
    lines += ["garbage line", _row("[N/A]", 900.0)]
    out = _summary(lines)
    assert out["sm_mhz"] == 1410
    assert out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]
    assert out["samples"] == 7 and out["samples_under_load"] == 5
    assert out["power_w_max"] == 990.0


def test_thermal_reasons_are_reported():
    lines = [_row(1200, 800.0, thermal="Active"), _row(1250, 820.0, sw_thermal="Active"), _row(1300, 810.0)]
    out = _summary(lines)
    assert out["reasons"] == ["hw_thermal_slowdown", "sw_thermal_slowdown"]
    assert out["sm_mhz"] == 1250


def test_no_load_uses_every_sample_and_na_power():
    out = _summary([_row(1965, "[N/A]"), _row(1900, 100.0), _row(1800, 150.0)])
    assert out["sm_mhz"] == 1900 and out["samples_under_load"] == 3 and out["reasons"] == []


def test_unsampled():
    out = _summary([])
    assert out == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
