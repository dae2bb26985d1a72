"""The bench line's roofline inputs that do not come from the GPU (CPU).

`roofline.traffic` is read from the committed ncu summary of the roofline
kernel, and the strong-scaling field quotes the fixed 64-sequence job's HBM
roofline; both must stay reproducible from the repository alone.
"""

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_roofline_traffic_comes_from_the_committed_profile(bench):
    traffic = bench.profile_traffic(bench.ROOFLINE_PROFILE)
    assert isinstance(traffic, int)
    # algorithmic bytes of the 64-row gate/up product: INT8 weights, float64
    # scales, INT8 rows in, float32 SiLU*up rows out
    D, F, B = 2048, 5632, 64
    algorithmic = 2 * F * D + 2 * F * 8 + B * D + B * F * 4
    # the weights dominate and are read once: DRAM traffic within 10%
    assert 0.9 * algorithmic <= traffic <= 1.1 * algorithmic


def test_profile_traffic_missing_file_is_none(bench, tmp_path):
    assert bench.profile_traffic(tmp_path / "absent.md") is None


def test_strong_scaling_roofline(bench):
    # (W + KV_64) / (W + KV_64 / N): every GPU streams all weights each step
    assert bench.strong_roofline(1) == pytest.approx(1.0)
    assert bench.strong_roofline(2) == pytest.approx(1.21, abs=0.01)
    assert bench.strong_roofline(4) == pytest.approx(1.35, abs=0.01)
    assert bench.strong_roofline(8) == pytest.approx(1.44, abs=0.01)
