"""Cross-check against the reference's own CUDA extension, compiled from its
source for sm_100a by oracle/build_ref.py into oracle/_ref (a checker
only).  The append operators must agree bit for bit (rotated q, exact ring,
INT8 codes, scales), the fused exact-tail merge within the reference
test's tolerance, and host validation must raise the same messages.
Skipped when the reference module was not built."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from pagegauge_b200.cache import rope_tables
from pagegauge_b200.runtime import load_append_extension, read_device_error

pytestmark = pytest.mark.gpu

REF_SO = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "page_gauge_append_ext_ref.so"


@pytest.fixture(scope="module")
def ref():
    if not REF_SO.is_file():
        pytest.skip("oracle/_ref was not built (no reference checkout at build time)")
    spec = importlib.util.spec_from_file_location("page_gauge_append_ext_ref", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16 if t.element_size() == 2 else torch.int8)


def _gauge_state(batch, exact_ppr, code_ppr, hkv=8):
    z = dict(device="cuda")
    return [torch.zeros(batch * exact_ppr, 16, hkv, 128, dtype=torch.float16, **z),
            torch.zeros(batch * exact_ppr, 16, hkv, 128, dtype=torch.float16, **z),
            torch.zeros(batch * code_ppr, 16, hkv, 128, dtype=torch.int8, **z),
            torch.zeros(batch * code_ppr, 16, hkv, 128, dtype=torch.int8, **z),
            torch.zeros(batch * code_ppr, hkv, dtype=torch.float16, **z),
            torch.zeros(batch * code_ppr, hkv, dtype=torch.float16, **z)]


@pytest.mark.parametrize("batch,prefix,tail,logical,dynamic", [
    (1, 0, 2, 5, False), (3, 1, 2, 6, True), (2, 3, 2, 8, False), (8, 0, 16, 3, True)])
def test_page_gauge_append_matches_reference_extension(cuda_lib, ref, batch, prefix, tail,
                                                       logical, dynamic):
    g = torch.Generator().manual_seed(1000 + batch)
    n = logical * 16
    cos, sin = (t.cuda() for t in rope_tables(n))
    q = (torch.randn(batch, 32, 128, generator=g)).half().cuda()
    keys = (torch.randn(n, batch, 8, 128, generator=g) * 2).half().cuda()
    values = torch.randn(n, batch, 8, 128, generator=g).half().cuda()
    kc = (torch.randn(batch, 8, 128, generator=g) * 0.5).half().cuda()
    vc = (torch.randn(batch, 8, 128, generator=g) * 0.1).half().cuda()
    ours, theirs = _gauge_state(batch, prefix + tail, logical), _gauge_state(batch, prefix + tail, logical)
    rq_o, rq_t = torch.empty_like(q), torch.empty_like(q)
    ext = load_append_extension()
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    for p in range(n):
        if dynamic:
            pos.fill_(p)
            ext.rope_append_page_gauge_dynamic(q, keys[p], values[p], cos, sin, pos, kc, vc, rq_o,
                                               *ours, prefix)
            ref.rope_append_page_gauge_dynamic(q, keys[p], values[p], cos, sin, pos, kc, vc, rq_t,
                                               *theirs, prefix)
        else:
            ext.rope_append_page_gauge(q, keys[p], values[p], cos[p].contiguous(),
                                       sin[p].contiguous(), kc, vc, rq_o, *ours, prefix, p)
            ref.rope_append_page_gauge(q, keys[p], values[p], cos[p].contiguous(),
                                       sin[p].contiguous(), kc, vc, rq_t, *theirs, prefix, p)
        if p % 7 == 0:
            assert torch.equal(_bits(rq_o), _bits(rq_t))
    torch.cuda.synchronize()
    assert read_device_error() == 0
    assert torch.equal(_bits(rq_o), _bits(rq_t))
    for a, b in zip(ours, theirs):
        assert torch.equal(_bits(a), _bits(b))


def test_fp16_append_matches_reference_extension(cuda_lib, ref):
    g = torch.Generator().manual_seed(77)
    batch, ppr = 4, 3
    cos, sin = (t.cuda() for t in rope_tables(ppr * 16))
    q = torch.randn(batch, 32, 128, generator=g).half().cuda()
    pages = [torch.zeros(batch * ppr, 16, 8, 128, dtype=torch.float16, device="cuda")
             for _ in range(4)]
    rq_o, rq_t = torch.empty_like(q), torch.empty_like(q)
    ext = load_append_extension()
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    for p in range(ppr * 16):
        k = torch.randn(batch, 8, 128, generator=g).half().cuda()
        v = torch.randn(batch, 8, 128, generator=g).half().cuda()
        if p % 2:
            ext.rope_append_fp16(q, k, v, cos[p].contiguous(), sin[p].contiguous(), rq_o,
                                 pages[0], pages[1], p)
            ref.rope_append_fp16(q, k, v, cos[p].contiguous(), sin[p].contiguous(), rq_t,
                                 pages[2], pages[3], p)
        else:
            pos.fill_(p)
            ext.rope_append_fp16_dynamic(q, k, v, cos, sin, pos, rq_o, pages[0], pages[1])
            ref.rope_append_fp16_dynamic(q, k, v, cos, sin, pos, rq_t, pages[2], pages[3])
        assert torch.equal(_bits(rq_o), _bits(rq_t))
    torch.cuda.synchronize()
    assert torch.equal(_bits(pages[0]), _bits(pages[2]))
    assert torch.equal(_bits(pages[1]), _bits(pages[3]))


@pytest.mark.parametrize("batch,tail_tokens", [(1, 1), (1, 16), (2, 17), (3, 255), (2, 256)])
def test_exact_tail_merge_matches_reference_extension(cuda_lib, ref, batch, tail_tokens):
    g = torch.Generator().manual_seed(500 + tail_tokens)
    n = 16
    q = torch.randn(batch, 32, 128, generator=g).half().cuda()
    ek = (torch.randn(batch * n, 16, 8, 128, generator=g) * 0.7).half().cuda()
    ev = torch.randn(batch * n, 16, 8, 128, generator=g).half().cuda()
    perm = torch.randperm(batch * n, generator=g).to(torch.int32).cuda()
    last = torch.full((batch,), (tail_tokens - 1) % 16 + 1, dtype=torch.int32, device="cuda")
    pages_used = -(-tail_tokens // 16)
    idx = torch.stack([perm[r * n:(r + 1) * n][:pages_used] for r in range(batch)]).reshape(-1)
    idx = idx.contiguous()
    old_o = torch.randn(batch, 32, 128, generator=g).half().cuda()
    old_l = (torch.randn(batch, 32, generator=g) * 3).float().cuda()
    vc = (torch.randn(batch, 8, 128, generator=g) * 0.1).half().cuda()
    o1, l1, o2, l2 = old_o.clone(), old_l.clone(), old_o.clone(), old_l.clone()
    load_append_extension().exact_tail_merge_center(q, ek, ev, idx, last, o1, l1, vc, 128 ** -0.5)
    ref.exact_tail_merge_center(q, ek, ev, idx, last, o2, l2, vc, 128 ** -0.5)
    torch.cuda.synchronize()
    # The reference's own tail-merge test tolerance (.py:671-676).
    torch.testing.assert_close(o1.float(), o2.float(), atol=3e-3, rtol=2e-3)
    torch.testing.assert_close(l1, l2, atol=2e-4, rtol=0)


def test_validation_messages_match_reference_extension(cuda_lib, ref):
    ext = load_append_extension()
    q = torch.zeros(2, 32, 128, dtype=torch.float16, device="cuda")
    k = torch.zeros(2, 8, 128, dtype=torch.float16, device="cuda")
    cos = torch.ones(128, dtype=torch.float16, device="cuda")
    pages = torch.zeros(4, 16, 8, 128, dtype=torch.float16, device="cuda")
    cases = [
        lambda m: m.rope_append_fp16(q.float(), k, k, cos, cos, q, pages, pages, 0),
        lambda m: m.rope_append_fp16(q, k[:1], k, cos, cos, q, pages, pages, 0),
        lambda m: m.rope_append_fp16(q, k, k, cos[:64], cos[:64], q, pages, pages, 0),
        lambda m: m.rope_append_fp16(q, k, k, cos, cos, q, pages, pages, -1),
        lambda m: m.rope_append_fp16(q, k, k, cos, cos, q, pages, pages, 16 * 4),
        lambda m: m.rope_append_fp16(q, k, k, cos, cos, q, pages, pages.transpose(1, 2), 0),
    ]
    for case in cases:
        with pytest.raises(RuntimeError) as ours:
            case(ext)
        with pytest.raises(RuntimeError) as theirs:
            case(ref)
        assert str(ours.value).splitlines()[0] in str(theirs.value), (ours.value, theirs.value)
