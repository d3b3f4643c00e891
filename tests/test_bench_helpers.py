"""bench.py's host-side accounting (CPU): the algorithmic bytes the roofline
uses per workload, the ragged workload's shapes and shards, and the exact
policy parser."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402


def test_algorithmic_bytes_known_answers():
    # B1/49K: 3,056 old pages + 256 exact tokens.
    assert bench.algorithmic_bytes([3056 * 16], [256]) == 101_285_376
    # B1/4K: 240 old pages + 256 exact tokens.
    assert bench.algorithmic_bytes([240 * 16], [256]) == 8_920_576
    # Per request the terms add: codes (K+V), scales (K+V), FP16 exact K+V.
    one = bench.algorithmic_bytes([16], [1])
    assert one == 2 * 16 * 8 * 128 + 1 * 8 * 2 * 2 + 2 * 1 * 8 * 128 * 2


def test_ragged_workload_is_seeded_and_sharded():
    mine, glob, shards = bench.workload_lengths("b8_ragged")
    assert len(glob) == 8 and mine == glob and shards == [list(range(8))]
    assert all(4096 <= n <= 32768 for n in glob)
    again = bench.workload_lengths("b8_ragged")
    assert again[1] == glob
    m0, g2, s2 = bench.workload_lengths("b8_ragged", world=2, rank=0)
    m1, _, _ = bench.workload_lengths("b8_ragged", world=2, rank=1)
    assert len(g2) == 16 and sorted(s2[0] + s2[1]) == list(range(16))
    assert sorted(m0 + m1) == sorted(g2)
    assert bench.workload_lengths("b1_49k", world=4) == ([49152], [49152] * 4, None)


def test_policy_parser():
    assert bench.parse_policy("S4/A0/T768") == (4, 0, 48)
    assert bench.parse_policy("S0/A0/T256") == (0, 0, 16)
    assert bench.parse_policy("S1/A128/T768") == (1, 128, 48)
    with pytest.raises(ValueError):
        bench.parse_policy("S0/A0/T250")
