"""CPU checks of the INT8 path's query decomposition (the kernel's int8
parts modelled by ``query_cases.split_query``): its per-element error bound,
and why it has three parts -- on queries with outlier channels a two-part
split leaves the decode outside the parity bar (max-abs 2e-3, base-2 LSE
2e-4) while three parts stay far inside it.  The GPU tests run the same
query kinds through the kernel (tests/test_gpu_outlier_q.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pagegauge_oracle as O
from pagegauge_b200.cache import synthetic_dense_cache

from query_cases import KINDS, outlier_queries, split_query

SM = 128 ** -0.5


@pytest.mark.parametrize("kind", ("gauss",) + KINDS)
def test_three_part_error_bound(kind):
    q = (torch.randn(4, 32, 128, generator=torch.Generator().manual_seed(2)).half()
         if kind == "gauss" else outlier_queries(4, 32, kind, seed=2))
    q = q.float().numpy()
    amax = np.abs(q).max(-1, keepdims=True)
    err3 = np.abs(split_query(q, 3) - q)
    err2 = np.abs(split_query(q, 2) - q)
    # sq/129032 from the last rounding, plus the FP32 rounding of the two
    # remainders (each within 2^-24 of amax): about amax * 1.8e-7 in all
    assert (err3 <= amax / 127 / 129032 + amax * 2.0 ** -23).all()
    assert (err2 <= amax / 127 / 508 * 1.01).all()


@pytest.fixture(scope="module")
def b1_4k():
    lengths = [4096]
    _, dk, dv = synthetic_dense_cache(lengths, seed=20261001)
    dk, dv = dk.numpy(), dv.numpy()
    ck = dk.reshape(-1, 8, 128).astype(np.float32).mean(0).astype(np.float16)
    cv = dv.reshape(-1, 8, 128).astype(np.float32).mean(0).astype(np.float16)
    codes_k, sk = O.quantize_pages_bulk(dk, ck)
    codes_v, sv = O.quantize_pages_bulk(dv, cv)
    ek = (dk[240:].astype(np.float32) - ck.astype(np.float32)).astype(np.float16)
    ev = (dv[240:].astype(np.float32) - cv.astype(np.float32)).astype(np.float16)
    return codes_k, codes_v, sk, sv, ek, ev, cv


def decode_with_split(q, case, parts):
    """B1/4K decode whose INT8 segment sees the split query and whose FP16
    tail sees the FP16 query, as in the kernel."""
    codes_k, codes_v, sk, sv, ek, ev, cv = case
    old = list(range(240))
    ko = O.dequant_tokens(codes_k, sk, old, 3840)
    vo = O.dequant_tokens(codes_v, sv, old, 3840)
    ke = O.gather_tokens(ek, list(range(16)), 256).astype(np.float64)
    ve = O.gather_tokens(ev, list(range(16)), 256).astype(np.float64)
    qs = q if parts == 0 else split_query(q, parts)
    out, lse = O.merge_states([O.attention_state(qs, ko, vo, SM), O.attention_state(q, ke, ve, SM)])
    return out + np.repeat(cv.astype(np.float64), 4, axis=0), lse


def test_two_parts_fail_outliers_three_parts_pass(b1_4k):
    two_parts_fail = []
    for kind in KINDS:
        q = outlier_queries(1, 32, kind, seed=5)[0].numpy()
        exp, exp_lse = decode_with_split(q, b1_4k, 0)
        o2, l2 = decode_with_split(q, b1_4k, 2)
        o3, l3 = decode_with_split(q, b1_4k, 3)
        # three parts: >20x inside the output bar, inside the LSE bar
        assert np.abs(o3 - exp).max() < 1e-4 and np.abs(l3 - exp_lse).max() < 2e-4, kind
        if np.abs(o2 - exp).max() > 2e-3 or np.abs(l2 - exp_lse).max() > 2e-4:
            two_parts_fail.append(kind)
    # Two parts break the bar on every outlier kind (x100: output 2.9e-3;
    # x300: LSE 2.5e-2).
    assert two_parts_fail == list(KINDS)
