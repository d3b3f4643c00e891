"""GPU parity of the affine_group16 representation (the reference's
alternative to PageGauge, scripts/benchmark_flashinfer_page_affine_int8.py:
166-189, :234-253, :567-602): the bulk quantiser bit-exact against the
oracle and the reference's own CPU output, and the decode (old affine pages,
optionally with an exact FP16 tail in the same launch or merged afterwards)
against the float64 oracle within max-abs 2e-3 and cosine >= 0.9999."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from pathlib import Path

from oracle import pagegauge_oracle as O
from pagegauge_b200 import wrapper as W
from pagegauge_b200.cache import synthetic_dense_cache
from pagegauge_b200.decode import PageGaugeDecode, split_tables
from pagegauge_b200.quantize import quantize_pages
from pagegauge_b200.runtime import read_device_error

from gpu_helpers import assert_close_decode, cpu

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
LSE_ATOL = 2e-4


def workspace(mb=64):
    return torch.empty(mb << 20, dtype=torch.uint8, device="cuda")


def test_quantiser_matches_reference_fixture(cuda_lib):
    g = np.load(GOLDEN / "quantize_affine_group16.npz")
    codes, bias, scale, recon = quantize_pages(torch.from_numpy(g["values"]).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(cpu(codes), g["codes"])
    assert np.array_equal(cpu(bias).view(np.uint16), g["bias"].view(np.uint16))
    assert np.array_equal(cpu(scale).view(np.uint16), g["scale"].view(np.uint16))
    assert np.array_equal(cpu(recon).view(np.uint16), g["reconstructed"].view(np.uint16))


@pytest.mark.parametrize("pages,heads,spread", [(97, 8, 0.35), (33, 2, 40.0), (5, 1, 1e-4)])
def test_quantiser_bit_exact_against_oracle(cuda_lib, pages, heads, spread):
    gen = torch.Generator().manual_seed(pages + heads)
    values = (torch.randn(pages, 16, heads, 128, generator=gen) * spread
              + torch.randn(heads, 128, generator=gen) * spread).half()
    codes, bias, scale, recon = quantize_pages(values.cuda())
    torch.cuda.synchronize()
    c, b, s, r = O.quantize_pages_affine(values.numpy())
    assert np.array_equal(cpu(codes), c)
    assert np.array_equal(cpu(bias).view(np.uint16), b.view(np.uint16))
    assert np.array_equal(cpu(scale).view(np.uint16), s.view(np.uint16))
    assert np.array_equal(cpu(recon).view(np.uint16), r.view(np.uint16))


def _affine_case(lengths, tail_pages, sink_pages=0, hkv=8, group=4, seed=20261003):
    q, dk, dv = synthetic_dense_cache(lengths, hkv=hkv, seed=seed, group=group)
    kc, kb, ks, _ = quantize_pages(dk.cuda())
    vc, vb, vs, _ = quantize_pages(dv.cuda())
    pages = [-(-n // 16) for n in lengths]
    tables = split_tables(pages, tail_pages, sink_pages)
    last = torch.tensor([(n - 1) % 16 + 1 for n in lengths], dtype=torch.int32, device="cuda")
    return q.cuda(), dk.cuda(), dv.cuda(), (kc, vc, kb, ks, vb, vs), tables, last


def _oracle(q, dk, dv, codes, tables, lengths, r):
    kc, vc, kb, ks, vb, vs = [cpu(t) for t in codes]
    o_ptr, o_idx, e_ptr, e_idx = tables
    old = o_idx[o_ptr[r]:o_ptr[r + 1]]
    ex = e_idx[e_ptr[r]:e_ptr[r + 1]]
    old_tok = 16 * len(old) if len(ex) else lengths[r]
    ex_tok = lengths[r] - old_tok
    return O.affine_decode(cpu(q[r]), kc, vc, kb, ks, vb, vs, old, old_tok, cpu(dk), cpu(dv), ex,
                           ex_tok)


@pytest.mark.parametrize("split", [0, 1, 5, 64])
@pytest.mark.parametrize("lengths", [[4096], [1000, 333, 2050, 17]])
def test_wrapper_old_pages_only(cuda_lib, lengths, split):
    """make_affine_wrapper over every page of ragged requests (partial last
    pages masked by last_page_len), as the reference's no-tail benchmark."""
    q, dk, dv, codes, _, last = _affine_case(lengths, 0)
    kc, vc, kb, ks, vb, vs = codes
    pages = [-(-n // 16) for n in lengths]
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(pages)]), dtype=torch.int32)
    indices = torch.arange(sum(pages), dtype=torch.int32, device="cuda")
    w = W.make_affine_wrapper(None, workspace())
    W.plan(w, indptr, indices, last, torch.int8, split)
    out, lse = w.run(q, (kc, vc), kb, ks, vb, vs, 128 ** -0.5, return_lse=True)
    torch.cuda.synchronize()
    assert read_device_error() == 0
    for r, n in enumerate(lengths):
        exp, exp_lse = O.affine_decode(cpu(q[r]), cpu(kc), cpu(vc), cpu(kb), cpu(ks), cpu(vb),
                                       cpu(vs), list(range(sum(pages[:r]), sum(pages[:r + 1]))), n)
        assert_close_decode(out[r], exp)
        np.testing.assert_allclose(cpu(lse[r]), exp_lse, atol=LSE_ATOL, rtol=0)


@pytest.mark.parametrize("hkv,group,warps", [(8, 4, 4), (2, 8, 2), (4, 1, 8), (1, 2, 1)])
def test_fused_with_exact_tail(cuda_lib, hkv, group, warps):
    """Old affine pages and an exact FP16 tail (plus sink pages) in one
    split launch + merge: the reference's affine exact-segments run
    (affine run, FP16 tail run, merge_state_in_place) in one plan."""
    lengths = [3000, 260, 700]
    q, dk, dv, codes, tables, last = _affine_case(lengths, 4, 1, hkv=hkv, group=group, seed=9)
    kc, vc, kb, ks, vb, vs = codes
    o_ptr, o_idx, e_ptr, e_idx = tables
    dec = PageGaugeDecode(workspace(), warps_per_cta=warps)
    dec.plan(o_ptr, torch.from_numpy(o_idx).cuda(), e_ptr, torch.from_numpy(e_idx).cuda(), last,
             hkv * group, hkv, old_split_pages=7, exact_split_pages=2)
    lse = torch.empty(len(lengths), hkv * group, device="cuda", dtype=torch.float32)
    out = dec.run(q, kc, vc, ks, vs, dk, dv, None, lse=lse, affine_bias=(kb, vb))
    torch.cuda.synchronize()
    assert read_device_error() == 0
    for r in range(len(lengths)):
        exp, exp_lse = _oracle(q, dk, dv, codes, tables, lengths, r)
        assert_close_decode(out[r], exp)
        np.testing.assert_allclose(cpu(lse[r]), exp_lse, atol=LSE_ATOL, rtol=0)


def test_segmented_sequence_equals_fused(cuda_lib):
    """Affine wrapper on the old pages + FP16 wrapper on the tail +
    merge_state_in_place equals the fused launch."""
    lengths = [2500, 1200]
    q, dk, dv, codes, tables, last = _affine_case(lengths, 16, seed=4)
    kc, vc, kb, ks, vb, vs = codes
    o_ptr, o_idx, e_ptr, e_idx = tables
    full = torch.full((len(lengths),), 16, dtype=torch.int32, device="cuda")
    a = W.make_affine_wrapper(None, workspace())
    W.plan(a, torch.from_numpy(o_ptr), torch.from_numpy(o_idx).cuda(), full, torch.int8, 0)
    out, lse = a.run(q, (kc, vc), kb, ks, vb, vs, 128 ** -0.5, return_lse=True)
    t = W.BatchDecodeWithPagedKVCacheWrapper(workspace(), "NHD")
    W.plan(t, torch.from_numpy(e_ptr), torch.from_numpy(e_idx).cuda(), last, torch.float16, 0)
    t_out, t_lse = t.run(q, (dk, dv), return_lse=True)
    W.merge_state_in_place(out, lse, t_out, t_lse)
    dec = PageGaugeDecode(workspace())
    dec.plan(o_ptr, torch.from_numpy(o_idx).cuda(), e_ptr, torch.from_numpy(e_idx).cuda(), last)
    fused = dec.run(q, kc, vc, ks, vs, dk, dv, None, affine_bias=(kb, vb))
    torch.cuda.synchronize()
    assert (out.float() - fused.float()).abs().max().item() < 2e-3
    for r in range(len(lengths)):
        exp, _ = _oracle(q, dk, dv, codes, tables, lengths, r)
        assert_close_decode(fused[r], exp)


def test_single_launch_and_graph_replay(cuda_lib):
    lengths = [5000, 900]
    q, dk, dv, codes, tables, last = _affine_case(lengths, 16, seed=12)
    kc, vc, kb, ks, vb, vs = codes
    o_ptr, o_idx, e_ptr, e_idx = tables
    dec = PageGaugeDecode(workspace())
    dec.plan(o_ptr, torch.from_numpy(o_idx).cuda(), e_ptr, torch.from_numpy(e_idx).cuda(), last,
             old_split_pages=20, exact_split_pages=4)
    out = torch.empty_like(q)
    ref = dec.run(q, kc, vc, ks, vs, dk, dv, None, affine_bias=(kb, vb)).clone()
    for kw in ({"fused_merge": True}, {"cluster": 4}):
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            dec.run(q, kc, vc, ks, vs, dk, dv, None, out=out, affine_bias=(kb, vb), **kw)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                dec.run(q, kc, vc, ks, vs, dk, dv, None, out=out, affine_bias=(kb, vb), **kw)
            out.zero_()
            graph.replay()
            graph.replay()
        torch.cuda.synchronize()
        assert (out.float() - ref.float()).abs().max().item() < 2e-3
        del graph
    assert read_device_error() == 0


def test_rejects_bad_metadata(cuda_lib):
    lengths = [64]
    q, dk, dv, codes, _, last = _affine_case(lengths, 0)
    kc, vc, kb, ks, vb, vs = codes
    w = W.make_affine_wrapper(None, workspace())
    W.plan(w, torch.tensor([0, 4], dtype=torch.int32), torch.arange(4, dtype=torch.int32, device="cuda"),
           last, torch.int8, 0)
    with pytest.raises(ValueError, match="k_bias must be"):
        w.run(q, (kc, vc), kb[:, :4].contiguous(), ks, vb, vs)
    with pytest.raises(ValueError, match="needs k_bias"):
        w.run(q, (kc, vc), ks, vs)
