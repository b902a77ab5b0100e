"""CPU: the roofline arithmetic behind bench.py's sweep records and its line's `roofline`.

Algorithmic bytes count every routed expert's weights and scales once, every routed row's
activation and intermediate bytes once and the output once; the speed-of-light time is the slower
of moving those bytes at the measured copy bandwidth and doing the FLOPs at the fp8 figure.  The
numbers below are worked out by hand from the layer's shapes (H = 7168, I = 2048)."""

import pytest

import bench


def test_per_expert_constants():
    assert bench.W13_BYTES == 29_360_128 and bench.W2_BYTES == 14_680_064
    assert bench.S13_BYTES == 7_168 and bench.S2_BYTES == 3_584
    assert bench.FLOP_PER_ASSIGN == 88_080_384


def test_gemm_bytes_one_token_one_expert():
    g1, g2 = bench.gemm_bytes({"active": 1, "rows": 1, "T": 1})
    # GEMM1: W13 + its scales, the token row and its 56 scales, the hi/lo row pair and 16 scales
    assert g1 == 29_360_128 + 7_168 + (7_168 + 224) + (4_096 + 64)
    # GEMM2: W2 + its scales, the hi/lo row pair and scales, one bf16 output row
    assert g2 == 14_680_064 + 3_584 + (4_096 + 64) + 14_336


def test_roofline_record_t1():
    peaks = {"hbm_gbs": 6400.0}
    f = {"active": 1, "rows": 1, "T": 1}
    r = bench.roofline_record(f, 1, 50.0, peaks, 3400.0)
    byts = sum(bench.gemm_bytes(f)) + 1 * (256 * 4 + 56 * 4)   # plus the logits and token scales
    assert r["bound"] == "hbm"
    assert r["floor_us"] == pytest.approx(byts / 6400e9 * 1e6, abs=0.05)
    assert r["hbm_frac"] == pytest.approx(byts / 50e-6 / 6400e9, abs=1e-3)
    assert r["sol_frac"] == pytest.approx(r["floor_us"] / 50.0, abs=2e-3)
    assert r["tokens_per_s"] == pytest.approx(20_000.0)


def test_roofline_record_prefill_is_tensor_bound():
    # 16,384 tokens routed to 28 experts, 14,551 rows: the FLOPs, not the bytes, set the floor
    f = {"active": 28, "rows": 14_551, "T": 16_384}
    r = bench.roofline_record(f, 16_384, 1_260.0, {"hbm_gbs": 6400.0}, 3400.0)
    assert r["bound"] == "tensor"
    assert r["floor_us"] == pytest.approx(14_551 * bench.FLOP_PER_ASSIGN / 3400e12 * 1e6, abs=0.1)
    assert r["fp8_frac"] == pytest.approx(14_551 * bench.FLOP_PER_ASSIGN / 1_260e-6 / 3400e12, abs=1e-3)
