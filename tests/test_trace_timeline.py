"""CPU: the traced build's per-K-block handoff timeline of the wide GEMMs, as trace.py reads it.

The traced kernels write clock64 stamps of CTA 0, row-major [row][K-block]: row 0 MMA thread has
a free accumulator, 1 its operand stage is full, 2 its MMAs and commits are issued, 3 the first
promotion warp sees the accumulator, 4 + w promotion warp w releases it.  These tests feed the
reader synthetic stamps with known intervals and check the medians it reports.
"""

import torch

from moe_swarm_b200 import trace as TR


def _stamps(n=200, period=1250, late=(1, 5), late_by=500):
    tl = torch.zeros(TR.TL_ROWS, TR.TL_KBS, dtype=torch.int64)
    for k in range(n):
        base = 10_000 + k * period
        tl[0, k] = base + 600
        tl[1, k] = base + 700
        tl[2, k] = base + 1200
        tl[3, k] = base + 1500
        for w in range(8):
            tl[4 + w, k] = base + 2100 + (late_by if w in late else 0)
    return tl


def test_timeline_medians():
    d = TR.timeline(_stamps())
    assert d["period"] == 1250.0
    assert d["mma_wait_acc"] == 650.0          # row 0 of K-block k+1 minus row 2 of K-block k
    assert d["mma_wait_stage"] == 100.0
    assert d["mma_issue"] == 500.0
    assert d["commit_to_promotion"] == 300.0
    assert d["promotion_to_last_release"] == 1100.0   # the late warps release 500 later
    assert d["release_vs_w4"] == [0.0, 500.0, 0.0, 0.0, 0.0, 500.0, 0.0, 0.0]
    assert d["kbs"] == 180                      # K-blocks after the first 20


def test_timeline_needs_enough_k_blocks():
    assert TR.timeline(_stamps(n=30)) is None   # fewer than 40 recorded K-blocks
    assert TR.timeline(torch.zeros(TR.TL_ROWS, TR.TL_KBS, dtype=torch.int64)) is None
