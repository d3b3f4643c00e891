"""GPU parity of the INT8 QK path on queries with outlier channels.

The INT8 segment splits each FP16 query row into int8 parts that share one
scale per row (``tests/query_cases.py``); the decomposition error grows
with the row's largest channel, so N(0,1) queries alone do not pin it.
Here Q rows carry 4 channels per head scaled x20 / x100 / x300, one
dominant channel over 0.01-scale noise, or three decades of per-channel
scale rotated by RoPE, and every query head is compared with the float64
oracle at the parity bar (max-abs 2e-3, cosine 0.9999; base-2 LSE 2e-4
plus 1e-6 relative, since outlier rows put the LSE in the hundreds)."""

from __future__ import annotations

import pytest

from gpu_helpers import check_all_heads, make_case
from query_cases import KINDS, outlier_queries
from test_gpu_decode import run_fused

pytestmark = pytest.mark.gpu


def check_heads(q, cache, tables, out, lse, request, group):
    check_all_heads(q, cache, tables, out, lse, request, group, lse_rtol=1e-6)


@pytest.mark.parametrize("kind", KINDS)
def test_b1_4k_outlier_queries_all_heads(cuda_lib, kind):
    q, dk, dv, cache, tables = make_case([4096], seed=20261001)
    q = outlier_queries(1, 32, kind, seed=11).cuda()
    out, lse, _ = run_fused(q, cache, tables, split_old=16)
    check_heads(q, cache, tables, out, lse, 0, 4)


@pytest.mark.parametrize("kind", ("x100", "dominant"))
def test_gqa8_outlier_queries(cuda_lib, kind):
    """GQA 8 runs the wide form of the split (a second MMA for the third
    part)."""
    q, dk, dv, cache, tables = make_case([3000, 1700], hkv=4, group=8, seed=9)
    q = outlier_queries(2, 32, kind, seed=12).cuda()
    out, lse, _ = run_fused(q, cache, tables, split_old=9, split_exact=4)
    for r in range(2):
        check_heads(q, cache, tables, out, lse, r, 8)


@pytest.mark.parametrize("kind", ("x300", "rope"))
def test_b1_49k_outlier_queries_all_heads(cuda_lib, kind):
    from pagegauge_b200 import scheduler

    q, dk, dv, cache, tables = make_case([49152], seed=20261002)
    q = outlier_queries(1, 32, kind, seed=13, position=49151).cuda()
    out, lse, _ = run_fused(q, cache, tables, split_old=scheduler.lookup(1, 49152))
    check_heads(q, cache, tables, out, lse, 0, 4)
