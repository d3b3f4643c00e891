"""Served cache layout host logic (CPU): page policy partition against the
production partition, capacity accounting known answers, request leases,
page closure and aging, decode metadata, and the pool views.  Mirrors the
reference's tests/test_serving_cpu_contract.py and
tests/test_serving_decode_metadata.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from pagegauge_b200 import serving as S
from pagegauge_b200.page_table import page_gauge_logical_partition


@pytest.mark.parametrize("suffix", [0, 128])
def test_partition_matches_production_partition(suffix):
    policy = S.Policy(4, suffix, 48)
    for prompt in (8192, 8193, 20480):
        for delta in (0, 1, 15, 16, 767, 768, 769, 1536):
            length = prompt + delta
            ours = S.partition(prompt, length, policy)
            prod = page_gauge_logical_partition((length + 15) // 16, 48, 4, (length - 1) % 16 + 1,
                                                suffix, prompt // 16)
            assert ours["history"] == prod["old_logical_pages"]
            assert ours["exact"] == prod["exact_logical_pages"]
            assert ours["history_tokens"] + ours["exact_tokens"] == length
            slots = [S.exact_slot(p, prompt, 2, policy) for p in ours["exact"]]
            assert len(set(slots)) == len(slots)
            assert all(2 * policy.storage_pages <= s < 3 * policy.storage_pages for s in slots)
    assert S.partition(8192, 8193)["tail_tokens"] == 753
    assert S.partition(8192, 8208)["tail_tokens"] == 768


def test_partition_errors():
    with pytest.raises(ValueError, match="Invalid prompt/current length"):
        S.partition(0, 10)
    with pytest.raises(ValueError, match="explicit FP16 fallback"):
        S.partition(128, 128)
    with pytest.raises(ValueError, match="Invalid page policy"):
        S.Policy(tail_pages=0)
    with pytest.raises(ValueError, match="Negative page"):
        S.exact_slot(-1, 8192, 0)


def test_lease_reuse_reorder_and_release():
    m = S.RequestSlots(2)
    a = m.admit("a", 8192, range(512))
    b = m.admit("b", 8200, range(1000, 1513))
    assert m.batch(["b", "a"]) == (b, a)
    assert m.state(b).current_tokens == 8200
    with pytest.raises(MemoryError):
        m.admit("c", 8192, range(2000, 2512))
    m.release(a)
    c = m.admit("c", 8192, range(512))
    assert c.slot == a.slot and c.generation > a.generation
    with pytest.raises(ValueError):
        m.state(a)
    with pytest.raises(ValueError):
        m.release(a)
    with pytest.raises(ValueError):
        m.append(b, 8192, range(1000, 1513))
    with pytest.raises(ValueError):
        m.batch(["c", "c"])


def test_append_closes_pages_and_ages_them():
    m = S.RequestSlots(2)
    a = m.admit("a", 8192, range(512))
    b = m.admit("b", 8192, range(2000, 2512))
    with pytest.raises(ValueError):
        m.append(a, 8192, list(range(512)) + [2000])  # b's page
    closed, aged = [], []
    for position in range(8192, 8192 + 800):
        ev = m.append(a, position, range((position + 16) // 16))
        if ev["closed_page"] is not None:
            closed.append(ev["closed_page"])
        aged.extend(ev["new_history_pages"])
    assert closed == list(range(512, 562))
    assert all(p < 562 for p in aged) and 512 in aged
    assert m.batch(["b", "a"]) == (b, a)


def test_accounting_known_answers_and_budget():
    ref = S.Layout(32, 4 * 1376, 4)
    assert ref.accounting()["total_served_capacity_bytes"] == 7288520704
    cand = S.Layout(32, 4 * 1376, 4, policy=S.Policy(4, 0, 48))
    assert cand.accounting()["total_served_capacity_bytes"] == 6214778880
    acc = ref.accounting()
    assert ref.admissible_pages(acc["total_served_capacity_bytes"]) == 4 * 1376
    with pytest.raises(MemoryError):
        ref.admissible_pages(acc["reserved_sidecar_bytes"] - 1)
    with pytest.raises(ValueError):
        S.RequestSlots(1).admit("short", 128, range(8))
    # A B200-sized budget: 180 GB minus 14.5 GB of weights and 8 GB reserved.
    lay = S.Layout.for_budget(32, 64, int(180e9 - 14.5e9 - 8e9))
    assert lay.accounting()["total_served_capacity_bytes"] <= 180e9 - 14.5e9 - 8e9
    assert S.Layout(32, lay.physical_pages + 1, 64).accounting()[
        "total_served_capacity_bytes"] > 180e9 - 14.5e9 - 8e9


def _manager():
    m = S.RequestSlots(2, S.Policy(suffix_pages=0))
    a = m.admit("a", 8192, range(512))
    b = m.admit("b", 8207, range(1000, 1513))
    return m, a, b


def test_decode_metadata_reorder_and_aging():
    m, a, b = _manager()
    batch = S.prepare_decode(m, [(b, 8207, range(1000, 1513)), (a, 8192, tuple(range(512)) + (2000,))])
    cols = batch.columns()
    assert cols["positions"] == (8207, 8192)
    assert cols["request_slots"] == (1, 0)
    assert cols["physical_token_slots"] == (1512 * 16 + 15, 2000 * 16)
    assert batch.rows[1].new_history_logical_pages == (464,)
    assert batch.rows[1].new_history_physical_pages == (464,)
    # Outgoing and incoming pages share a ring slot; the outgoing page's
    # codes were written when it closed, so the slot may be overwritten.
    assert batch.rows[1].new_history_exact_slots[0] == batch.rows[1].exact_token_slot // 16
    assert m.state(a).current_tokens == 8192
    S.commit_decode(m, batch)
    assert (m.state(a).current_tokens, m.state(b).current_tokens) == (8193, 8208)
    with pytest.raises(ValueError):
        S.commit_decode(m, batch)


def test_rejected_batch_does_not_advance():
    m, a, b = _manager()
    with pytest.raises(ValueError):
        S.prepare_decode(m, [(a, 8192, tuple(range(512)) + (2000,)), (b, 8208, range(1000, 1513))])
    assert m.state(a).current_tokens == 8192 and 2000 not in m.page_owner


def test_stale_generation_and_late_alias_rejected():
    m, a, b = _manager()
    batch = S.prepare_decode(m, [(a, 8192, tuple(range(512)) + (2000,))])
    m.release(a)
    m.admit("a", 8192, range(512))
    with pytest.raises(ValueError):
        S.commit_decode(m, batch)
    m, a, b = _manager()
    batch = S.prepare_decode(m, [(a, 8192, tuple(range(512)) + (2000,))])
    m.append(b, 8207, range(1000, 1513))
    m.append(b, 8208, tuple(range(1000, 1513)) + (2000,))
    with pytest.raises(ValueError):
        S.commit_decode(m, batch)


def test_decode_tables_cover_each_request_once():
    policy = S.Policy(1, 2, 4)
    m = S.RequestSlots(3, policy)
    rng = np.random.default_rng(1)
    free = [int(p) for p in rng.permutation(400)]
    leases = []
    for i, prompt in enumerate((200, 333, 517)):
        n = -(-prompt // 16)
        pages, free = free[:n], free[n:]
        leases.append(m.admit(f"r{i}", prompt, pages))
    sched = []
    for lease in leases:
        st = m.state(lease)
        pages = list(st.physical_pages)
        if st.current_tokens % 16 == 0:
            pages.append(free.pop())
        sched.append((lease, st.current_tokens, pages))
    batch = S.prepare_decode(m, sched)
    o_ptr, o_idx, e_ptr, e_idx, last, o_tok, e_tok = S.decode_tables(batch, policy)
    for r, row in enumerate(batch.rows):
        n_old, n_ex = o_ptr[r + 1] - o_ptr[r], e_ptr[r + 1] - e_ptr[r]
        assert o_tok[r] == 16 * n_old and o_tok[r] + e_tok[r] == row.position + 1
        assert (n_old + n_ex) == -(-(row.position + 1) // 16)
        ex = e_idx[e_ptr[r]:e_ptr[r + 1]]
        assert ex[-1] == row.exact_token_slot // 16  # current page last
        assert set(o_idx[o_ptr[r]:o_ptr[r + 1]]) <= set(row.physical_pages)
        assert last[r] == row.position % 16 + 1


def test_pool_views_are_zero_copy_planes():
    pages, heads = 6, 2
    codes = pages * 16 * heads * 128
    raw = torch.arange(2 * codes + 4 * pages * heads, dtype=torch.int64).remainder(251).to(torch.uint8)
    v = S.dense_pool_views(raw, pages, heads)
    assert v["key_codes"].shape == (pages, 16, heads, 128)
    assert v["value_scales"].shape == (pages, heads)
    assert v["key_codes"].data_ptr() == raw.data_ptr()
    assert v["value_codes"].data_ptr() == raw.data_ptr() + codes
    assert v["key_scales"].data_ptr() == raw.data_ptr() + 2 * codes
    engine = raw.view(pages, heads, 1, 2 * 16 * 128 + 4)
    w = S.from_engine_layer(engine, pages, heads)
    assert w["value_scales"].data_ptr() == v["value_scales"].data_ptr()
    with pytest.raises(ValueError, match="exact size"):
        S.dense_pool_views(raw[:-2], pages, heads)
    with pytest.raises(ValueError, match="copying is forbidden"):
        S.from_engine_layer(engine.float(), pages, heads)
    with pytest.raises(ValueError, match="Invalid physical pages"):
        S.zero_physical_pages(v, [0, 0])
    with pytest.raises(ValueError, match="CUDA"):
        S.zero_physical_pages(v, [1])
    lay = S.Layout(2, 8, 2, kv_heads=2, query_heads=4, policy=S.Policy(1, 1, 2))
    with pytest.raises(MemoryError):
        S.allocate_sidecars(lay, device="cpu", cache_budget_bytes=10)
    side = S.allocate_sidecars(lay, device="cpu",
                               cache_budget_bytes=lay.accounting()["total_served_capacity_bytes"])
    assert side["exact_key"].shape == (2, 2 * 4, 16, 2, 128)
