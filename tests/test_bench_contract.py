"""CPU checks of the measurement plumbing in bench.py: the clock sampler's
timed-region summary, the per-launch traffic figures the roofline objects
carry (equal to the profiles/ summaries'), the shared metric names of both
arms, and the profile summaries' commands (ncu always with
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


def _profile_traffic(name):
    for ln in (ROOT / "profiles" / f"{name}.md").read_text().splitlines():
        if ln.strip().startswith("traffic_bytes_per_launch:"):
            return int(float(ln.split(":", 1)[1]))
    return None


def test_roofline_traffic_matches_profiles(bench):
    """bench.py carries each per-launch traffic figure (it reads no profile at
    run time); every figure equals the one in the summary its comment names."""
    src = (ROOT / "bench.py").read_text()
    table = src.split("TRAFFIC = {", 1)[1].split("}", 1)[0]
    for line in table.strip().splitlines():
        key, rest = line.split(":", 1)
        key = key.strip().strip('"')
        assert "# profiles/" in rest, key
        prof = rest.split("# profiles/", 1)[1].split(".md", 1)[0]
        assert bench.TRAFFIC[key] == _profile_traffic(prof), (key, prof)


def test_both_arms_name_the_same_metric(bench):
    """The driver divides the two arms' values only when metric, unit and
    direction agree: both arms take the metric string from the same helper."""
    import inspect

    import torch

    assert bench.gemm_metric(32768, torch.bfloat16) == "GEMM TFLOP/s (M=N=K=32768, bfloat16)"
    ours = inspect.getsource(bench.run_gemm_spmd)
    ref = inspect.getsource(bench.reference_arm)
    assert '"metric": gemm_metric(n, dtype)' in ours and "gemm_metric(n, dt)" in ref
    assert "pair_metric(96, 2208, 6912)" in inspect.getsource(bench.run_ours)
    assert "pair_metric(96, 2208, 6912)" in ref
    assert "gemm_metric(n, torch.float32)" in ref and "torch.float32)" in inspect.getsource(bench.run_ours)


def test_pair_int8_ops_follow_the_kernel_form(bench):
    """The base-254 form: 10 products per K step of each 128 x 64 unit, naux
    padded to the 64-wide stage; naux past 33280 runs as K chunks of the same
    products."""
    ops = bench.pair_int8_ops(1176, 432, 1152)
    units = 7 + 5 + 3 + 1
    assert ops == 1176 * units * 2 * 10 * 64 * 128 * 1152 * 2.0
    assert bench.pair_int8_ops(1, 40, 33281) == 1 * 1 * 2 * 10 * 64 * 128 * 33344 * 2.0
    assert "read_traffic" not in (ROOT / "bench.py").read_text()


@pytest.mark.parametrize("path", sorted((ROOT / "profiles").glob("*.md")), ids=lambda p: p.name)
def test_profile_commands(path):
    text = path.read_text()
    assert "_work" not in text and "gpurun" not in text
    cmds = [ln.strip() for ln in text.splitlines() if ln.startswith("    ncu ")]
    assert cmds, "each summary gives the command that made it"
    for c in cmds:
        assert "--clock-control none" in c
        assert "python bench.py" in c
