"""bench.py's CPU-side pieces: the DRAM traffic it reports per launch comes
from the committed ncu summaries under profiles/ (per launch for config 2,
per update scaled to the launch for configs 3-5)."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config2_traffic_is_per_step():
    t = _bench()._profile_traffic("step_kernel_config2.txt")
    assert t is not None and 30e6 < t < 110e6  # 4096 envs x 25.5 KB at most


@pytest.mark.parametrize("name,units,lo,hi", [
    ("step_kernel_config3.txt", 262144, 15_000, 26_000),
    ("rollout_kernel_config4.txt", 32768 * 8, 15_000, 18_000),
    ("search_kernels_config5.txt", 64000 * 40, 1_000, 1_400),
])
def test_scaled_traffic_per_update(name, units, lo, hi):
    b = _bench()
    t = b._profile_traffic(name, units)
    assert t is not None and lo * units < t < hi * units
    assert b._profile_traffic(name, 2 * units) == pytest.approx(2 * t)


def test_profiles_name_their_commands():
    for f in sorted((ROOT / "profiles").glob("*.txt")):
        text = f.read_text()
        assert "Commands" in text and "ncu " in text and "--clock-control none" in text, f.name


def test_missing_profile_reports_no_traffic():
    assert _bench()._profile_traffic("no_such_profile.txt") is None
