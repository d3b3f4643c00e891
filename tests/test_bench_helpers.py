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


def test_ragged_workload_is_seeded_and_strongly_sharded():
    mine, glob, shards = bench.workload_lengths("b8_ragged")
    assert len(glob) == 8 and mine == glob and shards == [list(range(8))]
    assert all(4096 <= n <= 32768 for n in glob)
    again = bench.workload_lengths("b8_ragged")
    assert again[1] == glob
    # The same 8 requests at every GPU count (strong scaling).
    for world in (2, 4, 8):
        parts = [bench.workload_lengths("b8_ragged", world=world, rank=r) for r in range(world)]
        assert all(p[1] == glob for p in parts)
        assert sorted(sum(parts[0][2], [])) == list(range(8))
        assert sorted(n for p in parts for n in p[0]) == sorted(glob)
        if world == 8:
            assert all(len(p[0]) == 1 for p in parts)
    other = bench.workload_lengths("b8_ragged", seed=20261002)[1]
    assert other != glob and len(other) == 8
    assert bench.workload_lengths("b1_49k", world=4) == ([49152], [49152], None)


def test_both_arms_print_the_same_config():
    class Args:
        workload, layers = "b1_49k", 4

    cfg = bench.workload_config(Args, 1)
    assert cfg["lengths"] == [49152] and cfg["seeds"] == [20261001, 20261002, 20261003]
    assert "405 MB > 126 MB L2" in cfg["l2"]
    assert bench.workload_bytes([49152]) == 101_285_376
    assert bench.workload_config(Args, 1) == cfg
    Args.workload = "b8_ragged"
    assert "strong" in bench.workload_config(Args, 8)["parallelism"]


def test_policy_parser():
    assert bench.parse_policy("S4/A0/T768") == (4, 0, 48)
    assert bench.parse_policy("S0/A0/T256") == (0, 0, 16)
    assert bench.parse_policy("S1/A128/T768") == (1, 128, 48)
    with pytest.raises(ValueError):
        bench.parse_policy("S0/A0/T250")
