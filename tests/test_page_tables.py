"""Host page-table logic vs the reference's outputs (golden JSON produced
from the reference helpers) and the known answers its tests assert."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from pagegauge_b200 import page_table as PT
from pagegauge_b200.decode import split_tables

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "page_tables.json").read_text())


@pytest.mark.parametrize("case", GOLDEN["segment_page_table"])
def test_segment_page_table_matches_reference(case):
    rows, tail, sink = case["args"]
    out = PT.segment_page_table(rows, tail, sink, device="cpu")
    assert [t.tolist() for t in out] == case["out"]
    o_ptr, o_idx, e_ptr, e_idx = split_tables(rows, tail, sink)
    assert [o_ptr.tolist(), o_idx.tolist(), e_ptr.tolist(), e_idx.tolist()] == case["out"]


def test_segment_page_table_known_answer():
    """tests/test_flashinfer_page_affine_int8.py:50-57."""
    o_ptr, o_idx, e_ptr, e_idx = PT.segment_page_table([8, 6], tail_pages=2, sink_pages=1, device="cpu")
    assert o_ptr.tolist() == [0, 5, 8]
    assert o_idx.tolist() == [1, 2, 3, 4, 5, 9, 10, 11]
    assert e_ptr.tolist() == [0, 3, 6]
    assert e_idx.tolist() == [0, 6, 7, 8, 12, 13]


@pytest.mark.parametrize("case", GOLDEN["request_major_page_table"])
def test_request_major_page_table(case):
    b, p, phys = case["args"]
    assert PT.request_major_page_table(b, p, phys, device="cpu").tolist() == case["out"]


@pytest.mark.parametrize("case", GOLDEN["request_major_exact_page_table"])
def test_request_major_exact_page_table(case):
    assert PT.request_major_exact_page_table(*case["args"], device="cpu").tolist() == case["out"]


@pytest.mark.parametrize("case", GOLDEN["page_gauge_logical_partition"])
def test_logical_partition(case):
    part = PT.page_gauge_logical_partition(*case["args"])
    got = {k: (list(v) if isinstance(v, tuple) else v) for k, v in part.items()}
    assert got == case["out"]


def test_exact_sink_page_table_known_answer():
    """tests/test_page_gauge_transformer.py:126-151."""
    physical = PT.request_major_exact_page_table(2, 8, 2, 1, device="cpu")
    dest = torch.full((2, 3), -1, dtype=torch.int32)
    active = PT.write_exact_sink_tail_page_table(dest, physical, 6, 8, 1)
    assert physical.tolist() == [[0, 2, 1, 2, 1, 2, 1, 2], [3, 5, 4, 5, 4, 5, 4, 5]]
    assert active.tolist() == [[0, 1, 2], [3, 4, 5]]
    assert active.data_ptr() == dest.data_ptr()


def test_exact_prefix_s3_table_known_answer():
    """tests/test_page_gauge_transformer.py:154-183."""
    physical = PT.request_major_exact_page_table(2, 8, 2, 3, device="cpu")
    dest = torch.full((2, 5), -1, dtype=torch.int32)
    active = PT.write_exact_prefix_tail_page_table(dest, physical, 6, 8, 3)
    assert physical.tolist() == [[0, 1, 2, 4, 3, 4, 3, 4], [5, 6, 7, 9, 8, 9, 8, 9]]
    assert active.tolist() == [[0, 1, 2, 3, 4], [5, 6, 7, 8, 9]]


def test_partition_fails_closed():
    """tests/test_page_gauge_transformer.py:186-197."""
    with pytest.raises(ValueError, match="nonnegative integer"):
        PT.page_gauge_logical_partition(8, 2, -1, PT.PAGE)
    with pytest.raises(ValueError, match="quantized old page"):
        PT.page_gauge_logical_partition(3, 2, 1, PT.PAGE)
    with pytest.raises(ValueError, match="quantized old page"):
        PT.page_gauge_logical_partition(5, 2, 3, PT.PAGE)
    with pytest.raises(ValueError, match="segmented flashinfer_merge"):
        PT.validate_exact_prefix_attention_path(3, "fused_kernel")
    assert PT.validate_exact_prefix_attention_path(3, "flashinfer_merge") == 3


def test_heterogeneous_table_uses_old_then_ring():
    full = PT.request_major_page_table(2, 5, device="cpu")
    ring = PT.request_major_exact_page_table(2, 5, 2, device="cpu")
    dest = torch.full((2, 5), -1, dtype=torch.int32)
    out = PT.write_heterogeneous_page_table(dest, full, ring, 3, 5)
    assert out.tolist() == [[0, 1, 2, ring[0, 3].item(), ring[0, 4].item()],
                            [5, 6, 7, ring[1, 3].item(), ring[1, 4].item()]]


def test_exact_physical_index_agrees_with_table():
    table = PT.request_major_exact_page_table(3, 40, 16, 2, 4, 30, device="cpu")
    for r in range(3):
        for lp in range(40):
            assert PT.exact_physical_page_index(r, lp, 16, 2, 4, 30) == table[r, lp].item()


def test_old_page_table_follows_the_partition():
    """write_page_gauge_old_page_table gathers an exact-once old set (the
    partition's old pages with an exact prefix and a static suffix) from
    the request-major logical table, in logical order, with the reference's
    validation messages."""
    import torch

    from pagegauge_b200.page_table import (page_gauge_logical_partition,
                                           request_major_page_table,
                                           write_page_gauge_old_page_table)

    logical = request_major_page_table(3, 40, device="cpu")
    part = page_gauge_logical_partition(37, 8, 2, 5, 4, 30)
    old = part["old_logical_pages"]
    dest = torch.full((3, 40), -1, dtype=torch.int32)
    got = write_page_gauge_old_page_table(dest, logical, old)
    assert got.shape == (3, len(old))
    for r in range(3):
        assert got[r].tolist() == [r * 40 + p for p in old]
    assert (dest[:, len(old):] == -1).all()
    with pytest.raises(ValueError, match="unique and increasing"):
        write_page_gauge_old_page_table(dest, logical, (3, 2))
    with pytest.raises(ValueError, match="cannot be empty"):
        write_page_gauge_old_page_table(dest, logical, ())
    with pytest.raises(ValueError, match="exceeds allocated capacity"):
        write_page_gauge_old_page_table(dest, logical, (39, 40))
    with pytest.raises(ValueError, match="int32"):
        write_page_gauge_old_page_table(dest.long(), logical, old)
