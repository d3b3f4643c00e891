"""Property tests of the page-table helpers (host side, no GPU): for any
valid exact-page policy (S sink pages, A static-suffix pages, T tail-ring
pages) and context, the vectorised table equals the per-page index
function, the exact pages of a step occupy distinct slots of the request's
exact storage, and the logical partition covers every page exactly once."""

from __future__ import annotations

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from pagegauge_b200.page_table import (  # noqa: E402
    PAGE, exact_physical_page_index, page_gauge_logical_partition,
    request_major_exact_page_table)


@st.composite
def policies(draw):
    tail = draw(st.integers(1, 12))
    sink = draw(st.integers(0, 4))
    initial = draw(st.integers(sink + 2, sink + 40))
    suffix = draw(st.integers(0, initial - sink - 1))
    # The step's context: at least the prompt, with a quantized old page
    # left between the sink and the tail.
    total = draw(st.integers(max(initial, sink + tail + 1), initial + 60))
    return tail, sink, suffix, initial, total


@settings(max_examples=150, deadline=None)
@given(policies(), st.integers(1, 3))
def test_table_equals_index_function(policy, batch):
    tail, sink, suffix, initial, total = policy
    table = request_major_exact_page_table(batch, total, tail, sink, suffix, initial, device="cpu")
    for r in range(batch):
        for p in range(total):
            assert int(table[r, p]) == exact_physical_page_index(r, p, tail, sink, suffix, initial)


@settings(max_examples=150, deadline=None)
@given(policies(), st.integers(1, PAGE))
def test_exact_pages_of_a_step_have_distinct_slots(policy, last_len):
    tail, sink, suffix, initial, total = policy
    part = page_gauge_logical_partition(total, tail, sink, last_len, suffix, initial)
    exact = part["exact_logical_pages"]
    slots = [exact_physical_page_index(0, p, tail, sink, suffix, initial) for p in exact]
    # Fixed prefix / suffix slots and the tail ring never collide within a step,
    # and every slot lies inside the request's S + A + T exact pages.
    assert len(set(slots)) == len(slots)
    assert all(0 <= s < sink + suffix + tail for s in slots)


@settings(max_examples=150, deadline=None)
@given(policies(), st.integers(1, PAGE))
def test_partition_covers_every_page_once(policy, last_len):
    tail, sink, suffix, initial, total = policy
    part = page_gauge_logical_partition(total, tail, sink, last_len, suffix, initial)
    old, exact = part["old_logical_pages"], part["exact_logical_pages"]
    assert sorted(old + exact) == list(range(total))
    assert not set(old) & set(exact)
    assert part["tail_logical_pages"] == tuple(range(total - tail, total))
    assert part["context_token_count"] == (total - 1) * PAGE + last_len
    assert part["old_token_count"] == PAGE * len(old)
    assert part["exact_token_count"] == part["context_token_count"] - PAGE * len(old)
    assert len(old) >= 1
