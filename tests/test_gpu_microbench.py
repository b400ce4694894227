"""Sanity checks of the microbenchmarks the kernel design rests on
(tests/microbench/microbench.py): every MMA form completes, the measured
rates lie in a physically possible range, and the full-width M=128 f16 MMA
runs within reach of the nominal 4096 MACs per clock per SM."""

import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "microbench"))


@pytest.mark.gpu
def test_microbench_rates_are_sane():
    import microbench

    rows = microbench.run_all(quick=True)
    mma = [r for r in rows if r["what"].startswith("mma")]
    assert mma, rows
    for r in mma:
        # no tensor core does more than 8192 f16 MACs per clock per SM, and
        # a K=16 MMA never takes thousands of cycles
        assert 0 < r["mac_per_clk_sm"] <= 8192, r
        assert r["cycles_per_mma"] < 2000, r
    full = next(r for r in mma if r["what"] == "mma f16 A=smem M=128 N=256")
    assert full["mac_per_clk_sm"] > 2048, full
    for r in rows:
        if r["what"].startswith("issue"):
            assert 0 < r["lane_ops_per_clk_sm"] <= 256, r
