"""The bench line's roofline arithmetic on CPU: the largest kernel class against the peak it runs
closer to (`roofline`), and the whole timed region's algorithmic FLOPs against the sustained tensor
peak of all ranks (`step_roofline`), from a profile in the shape ge_profile returns."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PEAKS = {"hbm_gbs": 6550.7, "bf16_tflops": 1661.8, "bf16_tflops_sustained": 1396.2, "source": "measured"}
PROFILE = [
    {"name": "gemm_gate_up", "ms_per_launch": 0.05, "flops_per_launch": 6.9e10, "bytes_per_launch": 7.8e7,
     "launches_per_forward": 24},
    {"name": "residual_ffn", "ms_per_launch": 0.039, "flops_per_launch": 0.0, "bytes_per_launch": 2.1e8,
     "launches_per_forward": 24},
    {"name": "attention_sliding", "ms_per_launch": 0.035, "flops_per_launch": 2.2e10, "bytes_per_launch": 8.0e7,
     "launches_per_forward": 20},
]


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


def test_top_roofline_picks_the_largest_class_and_its_bound(bench):
    r = bench.top_roofline(PROFILE, PEAKS)
    assert r["kernel"] == "gemm_gate_up"
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert r["achieved"] == pytest.approx(6.9e10 / 0.05e-3 / 1e12)
    assert r["frac"] == pytest.approx(r["achieved"] / 1661.8)
    fwd_ms = 0.05 * 24 + 0.039 * 24 + 0.035 * 20
    assert r["share_of_forward"] == pytest.approx(0.05 * 24 / fwd_ms)


def test_top_roofline_of_a_byte_bound_class(bench):
    r = bench.top_roofline(PROFILE[1:2], PEAKS)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["achieved"] == pytest.approx(2.1e8 / 0.039e-3 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 6550.7)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_step_roofline_counts_every_rank(bench, world):
    steps, ms = 10, 100.0
    r = bench.step_roofline(PROFILE, PEAKS, steps, world, ms)
    flops = 6.9e10 * 24 + 2.2e10 * 20
    assert r["flop_per_forward"] == pytest.approx(flops)
    assert r["achieved"] == pytest.approx(flops * steps * world / (ms / 1000.0) / 1e12)
    assert r["peak"] == pytest.approx(1396.2 * world)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    assert r["peak_kind"] == "sustained bf16"
