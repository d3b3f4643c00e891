"""Zero-copy inputs: the batched append reads the new token's q/k/v
straight from page-locked host memory.  A CUDA graph of that call, replayed
after the host rewrote the rows, must see the new rows every time (the
kernel fetches them over the host link on every load, never a line an
earlier launch left in the L2).  Each replay's outputs (the rotated query
and the token written into the exact ring) must equal those of an eager
call on device copies of the same rows, with the loads after the
dependency wait (the default) or before it (``inputs_ready``, rows no
kernel writes)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("inputs_ready", [False, True])
def test_graph_replays_see_rewritten_host_rows(cuda_lib, inputs_ready):
    from pagegauge_b200.cache import build_gauge_cache, rope_tables, synthetic_dense_cache
    from pagegauge_b200.runtime import load_append_extension, read_device_error

    ext = load_append_extension()
    lengths = [300, 200]  # positions 299 / 199: no page closes
    _, dk, dv = synthetic_dense_cache(lengths, seed=20261001, device="cuda")
    # The batched append addresses request r's code pages at r * capacity.
    cache, _ = build_gauge_cache(dk, dv, lengths, capacity_pages=24)
    cos, sin = rope_tables(1024, device="cuda")
    positions = torch.tensor([n - 1 for n in lengths], dtype=torch.int32, device="cuda")
    B, hq, hkv = len(lengths), 32, 8
    hq_rows = torch.empty(B, hq, 128, dtype=torch.float16).pin_memory()
    hk_rows = torch.empty(B, hkv, 128, dtype=torch.float16).pin_memory()
    hv_rows = torch.empty(B, hkv, 128, dtype=torch.float16).pin_memory()
    rq = torch.empty(B, hq, 128, dtype=torch.float16, device="cuda")
    rq_ref = torch.empty_like(rq)

    def append(q, k, v, out, ready=False):
        ext.rope_append_page_gauge_batched(q, k, v, cos, sin, positions, cache.key_center,
                                           cache.value_center, out, cache.exact_key,
                                           cache.exact_value, cache.key_codes, cache.value_codes,
                                           cache.key_scales, cache.value_scales, 0,
                                           inputs_ready=ready)

    g = torch.Generator().manual_seed(7)
    for t in (hq_rows, hk_rows, hv_rows):
        t.copy_(torch.randn(t.shape, generator=g).half())
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        append(hq_rows, hk_rows, hv_rows, rq, inputs_ready)  # warm-up outside capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            append(hq_rows, hk_rows, hv_rows, rq, inputs_ready)
    torch.cuda.synchronize()
    ring_pages = [(n - 1) // 16 % 16 for n in lengths]
    for it in range(4):
        for t in (hq_rows, hk_rows, hv_rows):
            t.copy_(torch.randn(t.shape, generator=g).half())  # host writes
        graph.replay()
        torch.cuda.synchronize()
        assert read_device_error() == 0
        got_q = rq.clone()
        got_ring = [cache.exact_key[16 * r + ring_pages[r]].clone() for r in range(B)]
        append(hq_rows.cuda(), hk_rows.cuda(), hv_rows.cuda(), rq_ref)
        torch.cuda.synchronize()
        assert torch.equal(got_q, rq_ref), f"replay {it}: rotated query from stale host rows"
        for r in range(B):
            assert torch.equal(got_ring[r], cache.exact_key[16 * r + ring_pages[r]]), (it, r)
    assert read_device_error() == 0
    del graph
