"""The C-ABI library loads without a GPU, exports every symbol the header
declares, and its host-only planner produces the expected work lists."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from pagegauge_b200 import _lib
from pagegauge_b200.wrapper import plan_items

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from pagegauge_b200 import build

    build.build()
    return _lib.load()


def declared_symbols() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(pg_\w+)\s*\(", text, flags=re.M))
    return names


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert {"pg_decode_run", "pg_rope_append_page_gauge", "pg_exact_tail_merge_center"} <= names
    for name in names:
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTED) <= names


def test_struct_sizes_match_header_layout(lib):
    assert ctypes.sizeof(_lib.PgDecodeItem) == 16
    assert ctypes.sizeof(_lib.PgSegment) == 56
    sizes = (ctypes.c_int64 * 5)()
    assert lib.pg_struct_sizes(sizes, 5) == 0
    assert tuple(sizes) == (ctypes.sizeof(_lib.PgDecodeArgs), ctypes.sizeof(_lib.PgGemmArgs),
                            ctypes.sizeof(_lib.PgSegment), ctypes.sizeof(_lib.PgPlanInfo),
                            ctypes.sizeof(_lib.PgDecodeItem))
    assert lib.pg_abi_version() == 109


def test_planner_chunks_and_offsets(lib):
    indptr0 = np.array([0, 10, 10, 25], np.int32)   # request 1 has no old pages
    indptr1 = np.array([0, 2, 4, 5], np.int32)
    items, off, info = plan_items(3, 2, indptr0, indptr1, 4, 1, 148)
    # per head: r0: ceil(10/4)=3 old + 2 exact; r1: 0 + 2; r2: ceil(15/4)=4 + 1
    assert off.tolist() == [0, 5, 10, 12, 14, 19, 24]
    assert info.num_items == 24 and not info.single_item_per_head
    it = items.reshape(-1, 4)
    first = it[off[0]:off[1]]
    assert first[:, 0].tolist() == [0] * 5
    assert (first[:, 1] >> 16).tolist() == [0, 0, 0, 1, 1]
    assert first[:, 2].tolist() == [0, 4, 8, 0, 1]
    counts = first[:, 3] & 0x7FFFFFFF
    last_flag = (first[:, 3] >> 31) & 1
    assert counts.tolist() == [4, 4, 2, 1, 1]
    assert last_flag.tolist() == [0, 0, 1, 0, 1]
    # head 1 of request 0 is a copy with head index 1
    assert (it[off[1]:off[2], 1] & 0xFFFF).tolist() == [1] * 5


def test_planner_single_item_and_auto_split(lib):
    items, off, info = plan_items(1, 8, np.array([0, 100], np.int32), None, 1 << 20, 0, 148)
    assert info.single_item_per_head and info.num_items == 8
    # a fixed split above 32 pages per warp is capped (4 warps -> 128 pages)
    indptr = np.array([0, 3056], np.int32)
    items, off, info = plan_items(1, 8, indptr, None, 1 << 20, 0, 148)
    assert info.split_pages[0] == 128 and info.num_items == 8 * 24
    items, off, info = plan_items(1, 8, indptr, None, 0, 0, 148)
    # one full wave of 3 CTAs per SM (444 slots) with the smallest items
    assert info.split_pages[0] == 56
    assert info.num_items == 8 * -(-3056 // 56) <= 444
    # with the 16-page FP16 tail as one more item per head, 56 would need a
    # partial second wave (448 > 444): the planner moves to 57
    items, off, info = plan_items(1, 8, indptr, np.array([0, 16], np.int32), 0, 0, 148)
    assert info.split_pages[0] == 57 and info.num_items == 440


def test_planner_rejects_bad_input(lib):
    with pytest.raises(RuntimeError, match="non-decreasing"):
        plan_items(2, 8, np.array([0, 5, 3], np.int32), None, 4, 0, 148)
    with pytest.raises(RuntimeError, match="at least one segment"):
        plan_items(1, 8, None, None, 4, 0, 148)


def test_error_message_roundtrip_without_gpu(lib):
    rc = lib.pg_merge_state_in_place(None, None, None, None, -1, 128, 128, None)
    assert rc == 1
    assert b"non-negative" in lib.pg_last_error()


def test_tp_publish_validation_without_gpu(lib):
    peers = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    src = ctypes.c_void_p(0x30000)
    assert lib.pg_tp_publish(peers, 1, 0, 64, 64, 1, src, 4096, None) == 1
    assert b"world must be 2..8" in lib.pg_last_error()
    assert lib.pg_tp_publish(peers, 2, 0, 64, 65, 1, src, 4160, None) == 1
    assert b"tiles must be 1..tiles_cap" in lib.pg_last_error()
    assert lib.pg_tp_publish(peers, 2, 0, 64, 64, 33, src, 4096, None) == 1
    assert b"batch must be 1..32" in lib.pg_last_error()
    assert lib.pg_tp_publish(peers, 2, 0, 64, 64, 1, src, 4000, None) == 1
    assert b"src must be fp16" in lib.pg_last_error()


def test_tp_reduce_payload_validation_without_gpu(lib):
    ex = ctypes.c_void_p(0x10000)
    assert lib.pg_tp_reduce(ex, 2, 64, 64, 1, None, 0, None, 1e-5, ctypes.c_void_p(0x20000),
                            4096, 2, None) == 1
    assert b"payload must be PG_TP_PAYLOAD_F32" in lib.pg_last_error()


def _decode_items(items):
    it = items.reshape(-1, 4)
    return [(int(r), int(hs & 0xFFFF), int(hs >> 16), int(b), int(c & 0x7FFFFFFF), int((c >> 31) & 1))
            for r, hs, b, c in it]


def test_planner_every_page_exactly_once_ragged(lib):
    """Ragged requests (some without old or exact pages): per (request,
    head) the items of each segment tile its page range exactly once, in
    order, and the item ranges partition the list."""
    rng = np.random.default_rng(3)
    for batch in (1, 3, 8):
        old = rng.integers(0, 300, batch)
        old[0] = 0
        exact = rng.integers(0, 17, batch)
        if batch > 1:
            exact[1] = 0
        exact[0] = max(int(exact[0]), 1)  # every request has at least one page
        i0 = np.concatenate([[0], np.cumsum(old)]).astype(np.int32)
        i1 = np.concatenate([[0], np.cumsum(exact)]).astype(np.int32)
        for split0 in (0, 7, 64):
            items, off, info = plan_items(batch, 8, i0, i1, split0, 0, 148)
            decoded = _decode_items(items)
            assert off[0] == 0 and off[-1] == info.num_items == len(decoded)
            for r in range(batch):
                for h in range(8):
                    rh = r * 8 + h
                    mine = decoded[off[rh]:off[rh + 1]]
                    assert all(x[0] == r and x[1] == h for x in mine)
                    for seg, (lo, hi) in enumerate(((i0[r], i0[r + 1]), (i1[r], i1[r + 1]))):
                        runs = [(b, c, last) for _, _, s, b, c, last in mine if s == seg]
                        pos = lo
                        for b, c, last in runs:
                            assert b == pos and c > 0
                            pos += c
                        assert pos == hi
                        if runs:  # the last run of a segment carries the flag
                            assert [x[2] for x in runs] == [0] * (len(runs) - 1) + [1]


def test_planner_fixed_split_sizes_items(lib):
    indptr = np.array([0, 100], np.int32)
    items, off, info = plan_items(1, 8, indptr, None, 30, 0, 148)
    counts = [c for *_, c, _ in _decode_items(items)[:off[1]]]
    assert counts == [30, 30, 30, 10]
    assert info.split_pages[0] == 30


def test_gemm_default_grid_without_gpu(lib):
    """The streaming GEMM's default grid (seen through its scratch size,
    grid x segments x 64 x 8 floats): one CTA per SM for a narrow shape
    (<= 1024 weight blocks, e.g. a TP8 rank's qkv), every resident slot
    (3 per SM at one row) otherwise."""
    floats, tiles = ctypes.c_int64(0), ctypes.c_int32(0)
    # TP8 qkv: 12 tiles x 64 k-blocks = 768 blocks -> 148 CTAs, 2 segments each.
    assert lib.pg_skinny_gemm_workspace(768, 4096, 1, 0, 0, 148, ctypes.byref(floats),
                                        ctypes.byref(tiles)) == 0
    assert floats.value == 148 * 2 * 64 * 8
    # o at TP1: 64 tiles x 64 k-blocks = 4096 blocks -> 444 CTAs.
    assert lib.pg_skinny_gemm_workspace(4096, 4096, 1, 1, 0, 148, ctypes.byref(floats),
                                        ctypes.byref(tiles)) == 0
    assert floats.value == 444 * 2 * 64 * 8
    # An explicit grid is kept ...
    assert lib.pg_skinny_gemm_workspace(768, 4096, 1, 0, 100, 148, ctypes.byref(floats),
                                        ctypes.byref(tiles)) == 0
    assert floats.value == 100 * 2 * 64 * 8
    # ... unless more than 16 CTAs would share a tile (296 -> 153 here).
    assert lib.pg_skinny_gemm_workspace(768, 4096, 1, 0, 296, 148, ctypes.byref(floats),
                                        ctypes.byref(tiles)) == 0
    assert floats.value == 153 * 2 * 64 * 8
