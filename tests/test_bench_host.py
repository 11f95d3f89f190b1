"""bench.py's host-side accounting, on CPU: the algorithmic FLOP and byte
figures that its roofline and TFLOP/s fields divide by, the reference's token
stream and learning-rate schedule, and the parsing of the nvidia-smi clock
record that decides whether a run is kept.

FLOP figures are the scope table's per-step numbers: GPT-2 small B=8 T=1024
6.536 TFLOP (linears 1391.6 + causal attention 154.8 + LM head 632.4 GFLOP,
x3), tiny B=64 T=256 1.104 TFLOP, medium B=16 T=1024 37.22 TFLOP; GPT-2 XL
decode reads 6.224 GB of fp32 weights per step plus the K/V cache."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from oracle import oracle  # noqa: E402

XL_PARAMS = 1_557_611_200


def test_small_step_flops_match_the_scope_table():
    f = bench.step_flops(8, 1024)
    assert f["total"] == pytest.approx(6.536e12, rel=1e-3)
    assert f["attn"] / 3 == pytest.approx(154.8e9, rel=1e-3)
    assert f["gemm"] / 3 == pytest.approx((1391.6 + 632.4) * 1e9, rel=1e-3)
    # the per-config formula agrees with the small-model one
    assert bench.step_flops_cfg(12, 768, 50257, 8, 1024) == pytest.approx(f["total"], rel=1e-12)


@pytest.mark.parametrize("cfg,tflop", [((6, 384, 65, 64, 256), 1.104), ((24, 1024, 50257, 16, 1024), 37.22)])
def test_other_train_configs_flops(cfg, tflop):
    assert bench.step_flops_cfg(*cfg) / 1e12 == pytest.approx(tflop, rel=1e-3)


def test_xl_decode_bytes():
    # weights only at context 0; each cached position adds K and V of every layer
    assert bench.decode_bytes(XL_PARAMS, 48, 1600, 1, 0, 0) == pytest.approx(6.224e9, rel=2e-3)
    per_pos = 2 * 4 * 48 * 1600
    assert bench.decode_bytes(XL_PARAMS, 48, 1600, 8, 896, 128) - bench.decode_bytes(XL_PARAMS, 48, 1600, 8, 0, 0) \
        == pytest.approx(per_pos * 8 * (896 + 64))


def test_token_stream_and_schedule_follow_the_reference():
    assert np.array_equal(bench.lcg_tokens(4096, 50257, 12345), oracle.lcg_tokens(4096, 50257, 12345))
    t = bench.lcg_tokens(1 << 15, 50257, 12345)
    assert t.min() >= 0 and t.max() < 50257
    assert bench.lr_schedule(0) == pytest.approx(bench.LR / bench.WARMUP_LR)
    assert bench.lr_schedule(bench.WARMUP_LR - 1) == pytest.approx(bench.LR)
    assert bench.lr_schedule(bench.TOTAL_ITERS) == bench.LR_MIN


def test_clock_record_parsing():
    c = bench.ClockSampler(0)
    c.lines = list(enumerate([
        "0, 1950, 1965, 900.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 990.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1900, 1965, 999.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ]))
    s = c.summary()
    assert s["samples"] == 3 and s["sm_mhz"] == 1950 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    c.lines.append((4, "0, 1200, 1965, 700.0, 0x0000000000000008, Active, Not Active, Not Active, Not Active"))
    assert "hw_slowdown" in c.summary()["reasons"]


def test_clock_window_keeps_timed_samples():
    """Samples of the warm-up steps drop out once the timed region holds
    some; a region shorter than the sampling period keeps the warm-up's."""
    c = bench.ClockSampler(0)
    row = "0, {}, 1965, 900.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
    c.lines = [(0.0, row.format(1000)), (1.0, row.format(1900)), (1.2, row.format(1910))]
    c.mark(0.9, 1.1)
    s = c.summary()
    assert s["samples_in_window"] == 2 and s["samples"] == 2 and s["sm_mhz"] == 1905
    c.mark(5.0, 5.01)
    s = c.summary()
    assert s["samples_in_window"] == 0 and s["samples"] == 3


def test_step_gemm_shapes_cover_the_step():
    """The replayed GEMM list is the step's: 147 launches (12 per layer + the
    LM head's three) whose FLOPs are step_flops()'s GEMM part."""
    shapes = bench.step_gemm_shapes()
    assert len(shapes) == 12 * bench.L_ + 3 and len(set(shapes)) == 15
    assert sum(2.0 * M * N * K for (M, N, K, *_r) in shapes) == pytest.approx(bench.step_flops(8, 1024)["gemm"])
