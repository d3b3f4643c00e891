"""Ordering of a page close and the decode that reads the page as INT8.

Every kernel of this library lets the next kernel in the stream start
early (programmatic dependent launch), and the decode requests its INT8
tiles before it waits for the previous kernel.  That is correct while the
pages a decode reads as INT8 were closed at least one step earlier than
the kernels still running.  A one-page exact ring breaks that: the page
the append closes at step s is INT8 at step s+1, and a chain of early
starts can bring the next decode's tile requests ahead of the append's
code writes.  ``int8_after_wait`` makes the decode request the INT8 tiles
only after the previous kernel completes.  Here the decode launched right
behind the append reads the page that the append just closed, the
strongest form of the hazard, and must give the same bits as the same
launches with a host synchronisation in between, and match the oracle."""

from __future__ import annotations

import pytest
import torch

from pagegauge_b200.cache import build_gauge_cache, rope_tables, synthetic_dense_cache
from pagegauge_b200.decode import PageGaugeDecode
from pagegauge_b200.runtime import load_append_extension, read_device_error

from gpu_helpers import check_all_heads

pytestmark = pytest.mark.gpu

CAP = 48  # pages per request


def _case(layers, seed):
    # Request r holds 16*k_r + 15 tokens: its last page is one token short.
    ks = [5 + 4 * r for r in range(8)]
    lengths = [16 * k + 15 for k in ks]
    out = []
    g = torch.Generator().manual_seed(seed + 99)
    for layer in range(layers):
        q, dk, dv = synthetic_dense_cache(lengths, seed=seed + layer)
        cache, _ = build_gauge_cache(dk.cuda(), dv.cuda(), lengths, exact_tail_pages=1,
                                     capacity_pages=CAP)
        new = [torch.randn(8, n, 128, generator=g).half().cuda() for n in (32, 8, 8)]
        out.append((cache, new))
    return ks, lengths, out


def _run(ks, lengths, layers, synced):
    ext = load_append_extension()
    cos, sin = rope_tables(CAP * 16, device="cuda")
    positions = torch.tensor(lengths, dtype=torch.int32, device="cuda")  # token 15: closes
    indptr = torch.tensor([0] + list(torch.cumsum(torch.tensor([k + 1 for k in ks]), 0)),
                          dtype=torch.int32)
    indices = torch.cat([torch.arange(r * CAP, r * CAP + k + 1, dtype=torch.int32)
                         for r, k in enumerate(ks)]).cuda()
    dec = PageGaugeDecode(torch.empty(32 << 20, dtype=torch.uint8, device="cuda"))
    dec.plan(indptr, indices, None, None, None, 32, 8, old_split_pages=4)
    results = []
    for cache, (q, k, v) in layers:
        rq = torch.empty_like(q)
        out = torch.empty_like(q)
        lse = torch.empty(8, 32, dtype=torch.float32, device="cuda")
        ext.rope_append_page_gauge_batched(q, k, v, cos, sin, positions, cache.key_center,
                                           cache.value_center, rq, cache.exact_key,
                                           cache.exact_value, cache.key_codes, cache.value_codes,
                                           cache.key_scales, cache.value_scales, 0)
        if synced:
            torch.cuda.synchronize()
        dec.run(rq, cache.key_codes, cache.value_codes, cache.key_scales, cache.value_scales,
                None, None, cache.value_center, out=out, lse=lse, int8_after_wait=True)
        results.append((rq, out, lse, cache))
    torch.cuda.synchronize()
    assert read_device_error() == 0
    return results, indptr, indices


def test_decode_after_closing_append_reads_the_closed_page(cuda_lib):
    ks, lengths, layers_a = _case(4, 20261001)
    _, _, layers_b = _case(4, 20261001)
    fast, indptr, indices = _run(ks, lengths, layers_a, synced=False)
    slow, _, _ = _run(ks, lengths, layers_b, synced=True)
    for (rq1, o1, l1, c1), (rq2, o2, l2, c2) in zip(fast, slow):
        assert torch.equal(c1.key_codes, c2.key_codes)
        assert torch.equal(o1, o2) and torch.equal(l1, l2)

    class Tables:  # old segment only: pages 0..k_r, all full
        old_indptr, old_indices = indptr, indices
        exact_indptr = torch.zeros(9, dtype=torch.int32)
        exact_indices = torch.zeros(1, dtype=torch.int32)
        old_tokens = [16 * (k + 1) for k in ks]
        exact_tokens = [0] * 8

    rq, out, lse, cache = slow[-1]
    for r in range(8):
        check_all_heads(rq, cache, Tables, out, lse, r, 4)
