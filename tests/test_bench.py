"""Host-side logic of bench.py that the benchmark contract depends on (CPU):
the nvidia-smi clock-sample parsing, the device-index mapping under
CUDA_VISIBLE_DEVICES, the traffic figure read from the committed ncu summary,
and the shape of the profiles folder (text summaries that name their command).
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def sample(sm, mx=1965, reasons=("Not Active",) * 4, power=700.0):
    return ", ".join(["0", str(sm), str(mx), str(power), "0x0", *reasons])


def test_clock_summary_drops_first_sample_and_takes_median():
    cs = bench.ClockSampler(0)
    cs.lines = [sample(300), sample(1400), sample(1500), sample(1600)]
    s = cs.summary()
    assert s["samples"] == 3 and s["sm_mhz"] == 1500 and s["sm_max_mhz"] == 1965 and s["reasons"] == []


def test_clock_summary_reports_active_reasons():
    cs = bench.ClockSampler(0)
    cs.lines = [sample(1900),
                sample(1300, reasons=("Not Active", "Not Active", "Not Active", "Active")),
                sample(1200, reasons=("Active", "Not Active", "Not Active", "Active")),
                "garbled line"]
    s = cs.summary()
    assert s["samples"] == 2 and s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_summary_without_samples():
    cs = bench.ClockSampler(0)
    cs.lines = [sample(1900)]
    assert cs.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


@pytest.mark.parametrize("visible,index,expect", [("", 1, "1"), ("3,5", 1, "5"), ("GPU-abc, GPU-def", 0, "GPU-abc"),
                                                  ("2", 4, "4")])
def test_physical_device_index(monkeypatch, visible, index, expect):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", visible)
    assert bench.ClockSampler._physical(index) == expect


def test_traffic_read_from_committed_summary():
    t = bench.profile_traffic("window_attention_cfg2.md")
    assert t is not None and t > 0
    # within 2x of the algorithmic bytes of a 720p plain layer (packed Q/K/V read + output written)
    algorithmic = 23166 * 2560 * 3 * 2 + 21600 * 2560 * 2
    assert 0.5 * algorithmic < t < 2.0 * algorithmic
    assert bench.profile_traffic("no_such_summary.md") is None


def test_profiles_are_text_summaries_with_commands():
    pdir = os.path.join(ROOT, "profiles")
    names = sorted(os.listdir(pdir))
    assert names, "profiles/ is empty"
    for n in names:
        assert n.endswith((".md", ".txt")), f"profiles/{n}: only text summaries belong here"
        text = open(os.path.join(pdir, n)).read()
        assert "ncu " in text and "--clock-control none" in text, f"profiles/{n} does not give its ncu command"
        assert "<script" not in text, f"profiles/{n} names an uncommitted script"


def test_help_runs_without_a_gpu():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and "--cpu-euler" in r.stdout and "--impl" in r.stdout
