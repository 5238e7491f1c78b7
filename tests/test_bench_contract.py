"""CPU checks of the measurement plumbing in bench.py: the clock sampler's
timed-region summary, the per-launch traffic figures the roofline objects
read from profiles/, and the profile summaries' commands (ncu always with
--clock-control none, committed files only)."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_keeps_the_timed_region(bench):
    cs = bench.ClockSampler(0)
    cs.lines = [
        (1.0, "1900, 1965, 0x0000000000000001, 120"),  # idle, before the region
        (2.0, "1300, 1965, 0x0000000000000004, 990"),  # under load, power cap
        (2.2, "1320, 1965, 0x0000000000000004, 995"),
        (9.0, "1965, 1965, 0x0000000000000001, 100"),  # idle, after
    ]
    cs.start()
    cs.t0, cs.t1 = 1.5, 2.3
    s = cs.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1310.0
    assert s["reasons"] == ["sw_power_cap"] and s["sm_max_mhz"] == 1965.0
    # a region shorter than the sampling period keeps every sample
    cs.t0, cs.t1 = 5.0, 5.001
    assert cs.summary()["samples"] == 4


def test_roofline_traffic_profiles_exist(bench):
    names = set(bench.TRAFFIC_PROFILE.values()) | {"pair_energy_pair3"}
    for name in sorted(names):
        t = bench.read_traffic(name)
        assert isinstance(t, int) and t > 0, name


@pytest.mark.parametrize("path", sorted((ROOT / "profiles").glob("*.md")), ids=lambda p: p.name)
def test_profile_commands(path):
    text = path.read_text()
    assert "_work" not in text and "gpurun" not in text
    cmds = [ln.strip() for ln in text.splitlines() if ln.startswith("    ncu ")]
    assert cmds, "each summary gives the command that made it"
    for c in cmds:
        assert "--clock-control none" in c
        assert "python bench.py" in c
