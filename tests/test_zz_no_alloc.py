"""The allocation-free decode entry point (pg_decode_static).

Callers that cannot allocate device memory - a plugin living inside a host
process whose allocator owns the GPU, or a latency-critical path that must
not allocate - use pg_decode_static, whose scratch is a file-scope device
array inside the library.  This test calls it through the C ABI twice in a
row and checks both results against the workspace-based entry points
(pg_decode_plan + pg_decode_run) within the decode tolerance (max-abs 2e-3,
cosine >= 0.9999; LSE 2e-4).  It sits in its own file, collected last, and
builds all of its inputs itself so it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from pagegauge_b200 import _lib
from pagegauge_b200.decode import PageGaugeDecode
from pagegauge_b200.wrapper import _segment, host_indptr, num_sms

from gpu_helpers import assert_close_decode, make_case

pytestmark = pytest.mark.gpu


def _args(q, cache, tables, dec, out, lse):
    a = _lib.PgDecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
    a.batch, a.kv_heads, a.group = q.shape[0], 8, q.shape[1] // 8
    a.sm_scale = 128 ** -0.5
    a.seg[0] = _segment(cache.key_codes, cache.value_codes, tables.old_indices, dec._old_last,
                        cache.key_scales, cache.value_scales)
    a.seg[1] = _segment(cache.exact_key, cache.exact_value, tables.exact_indices,
                        tables.exact_last_page_len)
    a.warps_per_cta = 4
    a.out = out.data_ptr()
    a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
    a.lse_out = lse.data_ptr()
    a.value_center = cache.value_center.data_ptr()
    a.vc_stride_b = cache.value_center.stride(0)
    return a


def test_static_scratch_decode_matches_workspace_decode(cuda_lib):
    lengths = [4096, 2500, 700]
    q, dk, dv, cache, tables = make_case(lengths, seed=29)
    # Reference: the workspace-based entry points.
    dec = PageGaugeDecode(torch.empty(32 << 20, dtype=torch.uint8, device="cuda"))
    dec.plan(tables.old_indptr, tables.old_indices, tables.exact_indptr, tables.exact_indices,
             tables.exact_last_page_len, 32, 8, old_split_pages=9, exact_split_pages=4)
    ref_lse = torch.empty(3, 32, device="cuda", dtype=torch.float32)
    ref = dec.run(q, cache.key_codes, cache.value_codes, cache.key_scales, cache.value_scales,
                  cache.exact_key, cache.exact_value, cache.value_center, lse=ref_lse)
    torch.cuda.synchronize()
    ind0 = host_indptr(tables.old_indptr)
    ind1 = host_indptr(tables.exact_indptr)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.full((3, 32), float("nan"), device="cuda", dtype=torch.float32)
        a = _args(q, cache, tables, dec, out, lse)
        rc = lib.pg_decode_static(ctypes.byref(a), ind0.ctypes.data, ind1.ctypes.data, 9, 4,
                                  num_sms(q.device), stream)
        _lib.check(rc)
        torch.cuda.synchronize()
        for r in range(3):
            assert_close_decode(out[r], ref[r].float().cpu().numpy().astype(np.float64))
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=2e-4, rtol=0)


def test_static_scratch_rejects_plans_beyond_its_maximum(cuda_lib):
    q, dk, dv, cache, tables = make_case([2048], seed=31)
    dec = PageGaugeDecode(torch.empty(8 << 20, dtype=torch.uint8, device="cuda"))
    dec.plan(tables.old_indptr, tables.old_indices, tables.exact_indptr, tables.exact_indices,
             tables.exact_last_page_len, 32, 8)
    out = torch.empty_like(q)
    lse = torch.empty(1, 32, device="cuda", dtype=torch.float32)
    a = _args(q, cache, tables, dec, out, lse)
    # 65536 requests of one page each need more (request, head) pairs than
    # the static array plans for; the call is refused before any launch.
    a.batch = 65536
    big = np.arange(65537, dtype=np.int32)
    rc = _lib.load().pg_decode_static(ctypes.byref(a), big.ctypes.data, None, 1, 0, 148,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"at most" in _lib.load().pg_last_error()


def test_static_scratch_refuses_a_capturing_stream(cuda_lib):
    """Each call copies its plan from host memory, which a stream capture
    cannot record: the call is refused before anything is enqueued, and the
    caller's capture stays usable."""
    q, dk, dv, cache, tables = make_case([1024], seed=37)
    dec = PageGaugeDecode(torch.empty(8 << 20, dtype=torch.uint8, device="cuda"))
    dec.plan(tables.old_indptr, tables.old_indices, tables.exact_indptr, tables.exact_indices,
             tables.exact_last_page_len, 32, 8)
    out = torch.empty_like(q)
    lse = torch.empty(1, 32, device="cuda", dtype=torch.float32)
    a = _args(q, cache, tables, dec, out, lse)
    ind0 = host_indptr(tables.old_indptr)
    ind1 = host_indptr(tables.exact_indptr)
    lib = _lib.load()
    x = torch.zeros(16, device="cuda")
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        rc = lib.pg_decode_static(ctypes.byref(a), ind0.ctypes.data, ind1.ctypes.data, 0, 0,
                                  num_sms(q.device), stream.cuda_stream)
        x.add_(1)
    assert rc == 1
    assert b"being captured" in lib.pg_last_error()
    graph.replay()
    torch.cuda.synchronize()
    assert float(x[0]) == 1.0
