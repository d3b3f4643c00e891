"""Split scheduler host logic: buckets, the committed measured table, and
record/lookup round trips (no GPU)."""

from __future__ import annotations

from pagegauge_b200 import scheduler as S


def test_buckets_cover_half_octaves():
    assert S.bucket(1, 16384) == S.bucket(1, 24575) == "b1_c16384"
    assert S.bucket(1, 24576) == S.bucket(1, 32767) == "b1_c24576"
    assert S.bucket(1, 49152) == S.bucket(1, 65535) == "b1_c49152"
    assert S.bucket(1, 32768) == S.bucket(1, 49151) == "b1_c32768"
    assert S.bucket(8, 100) == S.bucket(8, 1535) == "b8_c1024"
    assert S.bucket(8, 3000) == "b8_c2048" and S.bucket(8, 3072) == "b8_c3072"


def test_committed_table_has_the_benchmark_shapes():
    entries = S.load_table()["entries"]
    for key in ("b1_c4096", "b1_c16384", "b1_c32768", "b1_c49152", "b8_c24576", "b32_c16384"):
        e = entries[key]
        assert e["split_pages"] == min(e["candidates_us"], key=lambda k: e["candidates_us"][k]) \
            or str(e["split_pages"]) == min(e["candidates_us"], key=e["candidates_us"].get)
        assert e["p50_us"] == min(e["candidates_us"].values())
    assert S.lookup(1, 49152) == entries["b1_c49152"]["split_pages"]
    assert all(e["mode"].startswith("steady") for e in entries.values())


def test_unmeasured_bucket_falls_back_to_heuristic(tmp_path):
    assert S.lookup(3, 5000, path=tmp_path / "none.json") == 0


def test_record_keeps_the_argmin(tmp_path):
    path = tmp_path / "t.json"
    assert S.record(2, 8192, {0: 12.0, 64: 10.5, 128: 11.0}, path=path) == 64
    assert S.lookup(2, 9000, path=path) == 64
    assert S.record(2, 8192, {0: 9.0, 64: 10.5}, path=path) == 0
    assert S.lookup(2, 8192, path=path) == 0


def test_candidates_span_one_to_64_splits():
    c = S.candidates(3056)
    assert c[0] == 0 and 48 in c and 64 in c
    assert all(-(-3056 // s) <= 64 for s in c if s)
    # sizes above the planner's 128-page cap collapse onto it
    assert max(c) == S.MAX_SPLIT_PAGES == 128 and 3056 not in c
    assert S.candidates(100) == sorted({0, 100, 50, 25, 13, 9, 7, 5, 4, 3, 2})


def test_refinements_surround_the_coarse_winner():
    from pagegauge_b200.scheduler import refinements

    assert refinements(0, [0, 64]) == []
    r = refinements(64, [0, 48, 55, 64, 77])
    assert r == [51, 54, 58, 61, 67, 70, 74]
    assert 77 not in r and 64 not in r


def test_kv_head_entries_and_fallback(tmp_path):
    path = tmp_path / "t.json"
    S.record(1, 16384, {24: 13.0, 48: 14.0}, path=path)
    # no entry of its own: the 8-head split scaled by kv_heads / 8
    assert S.lookup(1, 16384, path=path, kv_heads=2) == 6
    assert S.lookup(1, 16384, path=path, kv_heads=1) == 3
    # a measured entry for one head wins over the scaled fallback
    S.record(1, 16384, {3: 9.0, 12: 7.5}, path=path, kv_heads=1)
    assert S.lookup(1, 16384, path=path, kv_heads=1) == 12
    assert S.lookup(1, 16384, path=path) == 24
    assert S.bucket(1, 16384, 1) == "b1_c16384_h1" and S.bucket(1, 16384) == "b1_c16384"


def test_representation_entries_and_fallback(tmp_path):
    path = tmp_path / "t.json"
    S.record(1, 49152, {64: 20.0, 70: 19.5}, path=path)
    # affine_group16 without an entry of its own takes the page_gauge split
    assert S.lookup(1, 49152, path=path, representation="affine_group16") == 70
    S.record(1, 49152, {48: 24.0, 56: 23.0}, path=path, representation="affine_group16")
    assert S.lookup(1, 49152, path=path, representation="affine_group16") == 56
    assert S.lookup(1, 49152, path=path) == 70
    assert S.bucket(1, 49152, 8, "affine_group16") == "b1_c49152_affine"
    assert S.bucket(1, 49152, 2, "affine_group16") == "b1_c49152_h2_affine"
    # fewer heads: the representation's own 8-head entry, scaled
    assert S.lookup(1, 49152, path=path, kv_heads=4, representation="affine_group16") == 28
    import pytest
    with pytest.raises(ValueError):
        S.bucket(1, 49152, representation="fp8")
