"""The arithmetic behind bench.py's roofline object (no GPU): the dominant kernel, its work per
launch as the step's total work over its launch count, the achieved rate and fraction, and the
DRAM traffic scaled from the committed ncu capture."""
import importlib.util
import json
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0}


def test_roofline_tensor_kernel(bench):
    rows = 4096 * 128
    # 300 launches = 30 layers x 10 chunks, 330 us each
    prof = {"gemm_gateup_silu": (300 * 0.330, 300), "attention": (300 * 0.200, 300), "rmsnorm": (610 * 0.042, 610)}
    r = bench.roofline(prof, rows, PEAKS)
    assert r["kernel"] == "gemm_gateup_silu" and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    ops = 2 * (30 * rows * 3072 * 576 // 300)  # logical MACs per launch, 2 ops each
    assert r["ops_per_launch"] == ops
    assert r["launch_us"] == pytest.approx(330.0)
    assert r["achieved"] == pytest.approx(ops / 330e-6 / 1e12, rel=1e-3)
    assert r["peak"] == pytest.approx(2 * 1600.0)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"], rel=1e-3)
    assert r["rows_per_launch"] == rows * 30 // 300


def test_roofline_hbm_kernel(bench):
    rows = 4096 * 128
    prof = {"rmsnorm": (610 * 0.5, 610), "embed": (10 * 0.01, 10)}
    r = bench.roofline(prof, rows, PEAKS)
    assert r["kernel"] == "rmsnorm" and r["bound"] == "hbm" and r["unit"] == "GB/s"
    per_launch_bytes = 61 * rows * (576 * 4 + 576 * 2) // 610
    assert r["achieved"] == pytest.approx(per_launch_bytes / 500e-6 / 1e9, rel=1e-3)
    assert r["frac"] == pytest.approx(r["achieved"] / 6500.0, rel=1e-3)


def test_traffic_scales_with_rows(bench):
    with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
        t = json.load(f)
    e = t["gemm_gateup_silu"]
    assert bench.traffic_for("gemm_gateup_silu", e["rows"]) == e["dram_bytes"]
    assert bench.traffic_for("gemm_gateup_silu", 2 * e["rows"]) == 2 * e["dram_bytes"]
    assert bench.traffic_for("no_such_kernel", 128) is None


def test_roofline_named_kernel_and_tensor_activity(bench):
    rows = 4096 * 128
    prof = {"gemm_gateup_silu": (300 * 0.330, 300), "rmsnorm": (610 * 0.042, 610)}
    r = bench.roofline(prof, rows, PEAKS, kernel="rmsnorm")
    assert r["kernel"] == "rmsnorm" and r["bound"] == "hbm"
    d = bench.roofline(prof, rows, PEAKS)
    assert 0.0 < d["tensor_pipe_active_ncu"] < 1.0
