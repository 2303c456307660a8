"""The bench's clock sampler on the host, against a stand-in ``nvidia-smi``
(a shell script on PATH that prints rows in the real tool's CSV layout after
a start-up delay): a timed region shorter than the tool's start-up is still
sampled, rows written before the region are not counted as inside it, and
throttle reasons are read from the right columns."""
from __future__ import annotations

import os
import stat
import time

import pytest

import bench

ROW = "0, {mhz}, 1965, 900.5, 0x4, Not Active, Not Active, {thermal}, Active"


def _fake_smi(tmp_path, delay_s: float, period_s: float, mhz: int, thermal: str = "Not Active"):
    script = tmp_path / "nvidia-smi"
    script.write_text("#!/bin/bash\n"
                      f"sleep {delay_s}\n"
                      f"while true; do echo '{ROW.format(mhz=mhz, thermal=thermal)}'; sleep {period_s}; done\n")
    script.chmod(script.stat().st_mode | stat.S_IEXEC)
    return str(tmp_path)


@pytest.fixture
def fake_path(monkeypatch, tmp_path):
    def install(**kwargs):
        monkeypatch.setenv("PATH", _fake_smi(tmp_path, **kwargs) + os.pathsep + os.environ["PATH"])
    return install


def test_short_region_is_sampled_after_slow_start(fake_path):
    fake_path(delay_s=0.3, period_s=0.03, mhz=1800)
    with bench.ClockSampler(0) as sampler:
        time.sleep(0.15)  # shorter than the tool's start-up delay
    summary = sampler.summary()
    assert summary["samples"] >= 1
    assert summary["sm_mhz"] == 1800.0 and summary["sm_max_mhz"] == 1965.0
    assert summary["reasons"] == ["sw_power_cap"]
    assert "sampled" not in summary


def test_region_without_rows_reports_the_last_row_before_it(fake_path):
    fake_path(delay_s=0.0, period_s=5.0, mhz=1500)
    with bench.ClockSampler(0) as sampler:
        pass
    summary = sampler.summary()
    assert summary["samples"] == 0 and summary["sm_mhz"] == 1500.0
    assert "before the timed region" in summary["sampled"]


def test_thermal_slowdown_is_reported(fake_path):
    fake_path(delay_s=0.0, period_s=0.02, mhz=1200, thermal="Active")
    with bench.ClockSampler(0) as sampler:
        time.sleep(0.1)
    assert sampler.summary()["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_missing_tool_is_unsampled(monkeypatch, tmp_path):
    monkeypatch.setenv("PATH", str(tmp_path))
    with bench.ClockSampler(0) as sampler:
        pass
    assert sampler.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}


def test_mark_excludes_rows_before_the_region(fake_path):
    """Rows written between ``__enter__`` and ``mark()`` (a barrier between
    the ranks, in the bench) are not counted as inside the timed region."""
    fake_path(delay_s=0.0, period_s=0.02, mhz=1700)
    with bench.ClockSampler(0) as sampler:
        time.sleep(0.2)  # rows here belong to the barrier, not the region
        sampler.mark()
        marked = sampler.start_offset
        time.sleep(0.1)
    summary = sampler.summary()
    assert marked > 0
    assert 1 <= summary["samples"] <= 10  # ~5 rows at 20 ms in 0.1 s, none of the ~10 before mark()
