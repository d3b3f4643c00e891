"""Shared builders for the GPU parity tests: synthetic inputs on a CPU
generator (so the oracle and the GPU see the same bytes), caches built by
the product on the GPU, expected values from the CPU oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import pagegauge_oracle as O
from pagegauge_b200.cache import build_gauge_cache, synthetic_dense_cache

ATOL = 2e-3        # parity bar: max-abs 2e-3 in FP16 ...
MIN_COSINE = 0.9999  # ... and cosine >= 0.9999


def make_case(lengths, hkv=8, group=4, tail_pages=16, sink_pages=0, seed=20261001,
              capacity_pages=None):
    q, dk, dv = synthetic_dense_cache(lengths, hkv=hkv, seed=seed, group=group)
    cache, tables = build_gauge_cache(dk.cuda(), dv.cuda(), lengths, tail_pages, sink_pages,
                                      capacity_pages=capacity_pages)
    return q.cuda(), dk, dv, cache, tables


def cpu(t):
    return t.detach().cpu().numpy()


def check_quantizer_bit_exact(dk, dv, cache, lengths):
    """The GPU-built codes/scales equal the oracle's bulk quantiser given the
    same centres (fp32 centring, half-away rounding)."""
    pages = [-(-n // 16) for n in lengths]
    start = 0
    for r, n in enumerate(pages):
        for dense, codes, scales, center in ((dk, cache.key_codes, cache.key_scales, cache.key_center),
                                             (dv, cache.value_codes, cache.value_scales, cache.value_center)):
            c, s = O.quantize_pages_bulk(cpu(dense[start:start + n]), cpu(center[r]), "half_away")
            assert np.array_equal(cpu(codes[start:start + n]), c)
            assert np.array_equal(cpu(scales[start:start + n]).view(np.uint16), s.view(np.uint16))
        start += n


def oracle_decode(q, cache, tables, lengths, request, with_center=True, sm_scale=128 ** -0.5):
    o_ptr = cpu(tables.old_indptr)
    e_ptr = cpu(tables.exact_indptr)
    old_ids = cpu(tables.old_indices)[o_ptr[request]:o_ptr[request + 1]]
    ex_ids = cpu(tables.exact_indices)[e_ptr[request]:e_ptr[request + 1]]
    return O.page_gauge_decode(
        cpu(q[request]), cpu(cache.key_codes), cpu(cache.value_codes), cpu(cache.key_scales),
        cpu(cache.value_scales), old_ids, tables.old_tokens[request], cpu(cache.exact_key),
        cpu(cache.exact_value), ex_ids, tables.exact_tokens[request],
        cpu(cache.value_center[request]) if with_center else None, sm_scale)


def assert_close_decode(out, expected, atol=ATOL):
    got = out.float().cpu().numpy()
    err = O.max_abs(got, expected)
    cos = O.cosine(got, expected)
    assert err <= atol and cos >= MIN_COSINE, f"max-abs {err:.3e}, cosine {cos:.6f}"
    return err, cos


def check_all_heads(q, cache, tables, out, lse, request, group, lse_rtol=0.0):
    """Every KV head's query rows of ``request`` against the float64 oracle
    (one head at a time, so long contexts stay small on the host):
    outputs at the parity bar, base-2 LSE within 2e-4 (+ lse_rtol)."""
    ck, cv = cpu(cache.key_codes), cpu(cache.value_codes)
    sk, sv = cpu(cache.key_scales), cpu(cache.value_scales)
    ek, ev = cpu(cache.exact_key), cpu(cache.exact_value)
    o_ptr, e_ptr = cpu(tables.old_indptr), cpu(tables.exact_indptr)
    old_ids = cpu(tables.old_indices)[o_ptr[request]:o_ptr[request + 1]]
    ex_ids = cpu(tables.exact_indices)[e_ptr[request]:e_ptr[request + 1]]
    worst = 0.0
    for h in range(ck.shape[2]):
        hs = slice(h, h + 1)
        rows = slice(group * h, group * h + group)
        exp, exp_lse = O.page_gauge_decode(
            cpu(q[request, rows]), ck[:, :, hs], cv[:, :, hs], sk[:, hs], sv[:, hs], old_ids,
            tables.old_tokens[request], ek[:, :, hs], ev[:, :, hs], ex_ids,
            tables.exact_tokens[request], cpu(cache.value_center[request, hs]), 128 ** -0.5)
        err, _ = assert_close_decode(out[request, rows], exp)
        worst = max(worst, err)
        if lse is not None:
            np.testing.assert_allclose(cpu(lse[request, rows]), exp_lse, atol=2e-4, rtol=lse_rtol)
    return worst
