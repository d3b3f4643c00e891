"""GPU parity of the served pool (PageGauge kernels on a paged serving
layout with an S/A/T policy): prompt packing bit-exact against the oracle's
bulk quantiser, then decode steps driven by the request leases and decode
metadata -- rotated q and the new exact token bit-exact, closed pages'
codes bit-exact against the append rule, and the attention output within
max-abs 2e-3 / cosine 0.9999 of the float64 oracle over the pool's history
pages and the sidecar's exact pages."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pagegauge_oracle as O
from pagegauge_b200 import _lib
from pagegauge_b200 import serving as S
from pagegauge_b200.cache import rope_tables
from pagegauge_b200.runtime import read_device_error

from gpu_helpers import assert_close_decode, cpu

pytestmark = pytest.mark.gpu

HKV, HQ, D = 2, 8, 128


def _setup(prompts, policy, pages=300, layers=2, seed=3):
    lay = S.Layout(layers, pages, 4, kv_heads=HKV, query_heads=HQ, policy=policy)
    pool = S.ServedPool(lay)
    m = S.RequestSlots(4, policy)
    gen = torch.Generator().manual_seed(seed)
    free = [int(p) for p in torch.randperm(pages, generator=gen)]
    leases, raw = [], {}
    for i, prompt in enumerate(prompts):
        n = -(-prompt // 16)
        leases.append(m.admit(f"r{i}", prompt, free[:n]))
        free = free[n:]
        st = m.state(leases[-1])
        for layer in range(layers):
            k = (torch.randn(prompt, HKV, D, generator=gen) + 0.5).half()
            v = torch.randn(prompt, HKV, D, generator=gen).half()
            raw[(i, layer)] = (k.numpy(), v.numpy())
            pool.pack_prompt(layer, st, k.cuda(), v.cuda())
    torch.cuda.synchronize()
    return lay, pool, m, leases, free, gen, raw


def _check_prompt_packing(pool, m, leases, raw, layer=0):
    """Complete prompt pages: the bulk quantiser's codes (FP32 centring) in
    their physical pages; exact pages: f16(k - c) in their sidecar slots."""
    views = pool.views[layer]
    sc = pool.sidecars
    policy = pool.layout.policy
    for i, lease in enumerate(leases):
        st = m.state(lease)
        T = st.prompt_tokens
        n = -(-T // 16)
        for name, center, codes, scales, exact, x in (
                ("k", "key_center", "key_codes", "key_scales", "exact_key", raw[(i, layer)][0]),
                ("v", "value_center", "value_codes", "value_scales", "exact_value", raw[(i, layer)][1])):
            c = cpu(sc[center][layer, lease.slot])
            padded = np.zeros((n * 16, HKV, D), np.float16)
            padded[:T] = x
            paged = padded.reshape(n, 16, HKV, D)
            complete = T // 16
            z, s = O.quantize_pages_bulk(paged[:complete], c, "half_away")
            phys = list(st.physical_pages[:complete])
            assert np.array_equal(cpu(views[codes])[phys], z), name
            assert np.array_equal(cpu(views[scales])[phys].view(np.uint16), s.view(np.uint16)), name
            ex = cpu(sc[exact][layer])
            for lp in S.partition(T, T, policy)["exact"]:
                slot = S.exact_slot(lp, T, lease.slot, policy)
                want = (paged[lp].astype(np.float32) - c.astype(np.float32)).astype(np.float16)
                valid = min(16, T - 16 * lp)
                want[valid:] = 0
                assert np.array_equal(ex[slot].view(np.uint16), want.view(np.uint16)), (name, lp)


@pytest.mark.parametrize("policy", [S.Policy(1, 2, 4), S.Policy(0, 0, 3), S.Policy(2, 0, 6)])
def test_served_decode_matches_oracle(cuda_lib, policy):
    prompts = [200, 333, 517]
    lay, pool, m, leases, free, gen, raw = _setup(prompts, policy)
    for layer in range(lay.layers):
        _check_prompt_packing(pool, m, leases, raw, layer)
    cos, sin = rope_tables(1024, device="cuda")
    cos_h, sin_h = cpu(cos), cpu(sin)
    sm = 128 ** -0.5
    for step in range(40):
        sched = []
        order = [2, 0, 1] if step % 2 else [0, 1, 2]  # rows reordered between steps
        for i in order:
            st = m.state(leases[i])
            pages = list(st.physical_pages)
            if st.current_tokens % 16 == 0:
                pages.append(free.pop())
            sched.append((leases[i], st.current_tokens, pages))
        batch = S.prepare_decode(m, sched)
        pool.plan(batch, old_split_pages=3, exact_split_pages=2)
        o_ptr, o_idx, e_ptr, e_idx, _ = pool.tables
        B = len(batch.rows)
        for layer in range(lay.layers):
            qkv = torch.randn(B, (HQ + 2 * HKV) * D, generator=gen).half().cuda()
            q = qkv[:, :HQ * D].view(B, HQ, D)
            k = qkv[:, HQ * D:(HQ + HKV) * D].view(B, HKV, D)
            v = qkv[:, (HQ + HKV) * D:].view(B, HKV, D)
            rq = torch.empty(B, HQ, D, dtype=torch.float16, device="cuda")
            out = pool.step(layer, q, k, v, cos, sin, rq)
            torch.cuda.synchronize()
            views = pool.views[layer]
            sc = pool.sidecars
            codes_k, codes_v = cpu(views["key_codes"]), cpu(views["value_codes"])
            sk, sv = cpu(views["key_scales"]), cpu(views["value_scales"])
            ek, ev = cpu(sc["exact_key"][layer]), cpu(sc["exact_value"][layer])
            for r, row in enumerate(batch.rows):
                pos = row.position
                exp_q = O.rope_fp16(cpu(q[r]), cos_h[pos], sin_h[pos])
                assert np.array_equal(cpu(rq[r]).view(np.uint16), exp_q.view(np.uint16))
                ck = cpu(sc["key_center"][layer, row.lease.slot])
                cv = cpu(sc["value_center"][layer, row.lease.slot])
                ring = row.exact_token_slot // 16
                tok = pos % 16
                exp_k = (O.rope_fp16(cpu(k[r]), cos_h[pos], sin_h[pos]).astype(np.float32)
                         - ck.astype(np.float32)).astype(np.float16)
                assert np.array_equal(ek[ring, tok].view(np.uint16), exp_k.view(np.uint16))
                if tok == 15:  # the page closed: its codes are the append rule's
                    code_page = row.physical_token_slot // 16
                    for ring_pages, codes, scales in ((ek, codes_k, sk), (ev, codes_v, sv)):
                        centred = ring_pages[ring].astype(np.float32)
                        s = O.page_scale(np.abs(centred).max(axis=(0, 2)))
                        z = O.quantize_codes(centred, s[None, :, None], "half_away")
                        assert np.array_equal(codes[code_page], z)
                        assert np.array_equal(scales[code_page].view(np.uint16), s.view(np.uint16))
                old = o_idx[o_ptr[r]:o_ptr[r + 1]]
                ex = e_idx[e_ptr[r]:e_ptr[r + 1]]
                exp, _ = O.page_gauge_decode(cpu(rq[r]), codes_k, codes_v, sk, sv, old,
                                             pool.old_tokens[r], ek, ev, ex, pool.exact_tokens[r],
                                             cv, sm)
                assert_close_decode(out[r], exp)
        S.commit_decode(m, batch)
    assert read_device_error() == 0
    assert all(m.state(lease).current_tokens == p + 40 for lease, p in zip(leases, prompts))


def test_zero_pages_and_bad_slots(cuda_lib):
    policy = S.Policy(1, 2, 4)
    lay, pool, m, leases, free, gen, _ = _setup([200], policy, layers=1)
    views = pool.views[0]
    st = m.state(leases[0])
    victim = list(st.physical_pages[:3])
    S.zero_physical_pages(views, victim)
    torch.cuda.synchronize()
    for name in ("key_codes", "value_codes", "key_scales", "value_scales"):
        assert int(views[name][victim].abs().sum()) == 0
    assert int(views["key_codes"][list(st.physical_pages[3:12])].abs().sum()) > 0
    # A slot whose token disagrees with the position is skipped and reported.
    cos, sin = rope_tables(512, device="cuda")
    q = torch.randn(1, HQ, D, device="cuda").half()
    k = torch.randn(1, HKV, D, device="cuda").half()
    rq = torch.zeros_like(q)
    before = pool.sidecars["exact_key"].clone()
    dev32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")  # noqa: E731
    pos, ts, es, cr = dev32([200]), dev32([free[0] * 16 + 3]), dev32([5 * 16 + 8]), dev32([0])
    sc = pool.sidecars
    center_out = torch.empty(1, HKV, D, dtype=torch.float16, device="cuda")
    _lib.call("pg_rope_append_page_gauge_served", q.data_ptr(), k.data_ptr(), k.data_ptr(),
              cos.data_ptr(), sin.data_ptr(), sc["key_center"][0].data_ptr(),
              sc["value_center"][0].data_ptr(), rq.data_ptr(), sc["exact_key"][0].data_ptr(),
              sc["exact_value"][0].data_ptr(), views["key_codes"].data_ptr(),
              views["value_codes"].data_ptr(), views["key_scales"].data_ptr(),
              views["value_scales"].data_ptr(), center_out.data_ptr(), q.stride(0), k.stride(0),
              k.stride(0), 1, HQ, HKV, lay.physical_pages, sc["exact_key"].shape[1],
              sc["key_center"].shape[1], pos.data_ptr(), ts.data_ptr(), es.data_ptr(),
              cr.data_ptr(), cos.stride(0), cos.shape[0], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert read_device_error() == 3  # PG_DEV_BAD_PAGE_ID
    assert torch.equal(before, pool.sidecars["exact_key"])
