"""Pin the CPU oracle to fixtures produced by the reference itself
(tests/golden/make_golden.py) and to the reference tests' known answers."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import pagegauge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_quantize_page_gauge_codes_and_scales_bit_exact():
    g = np.load(GOLDEN / "quantize_page_gauge.npz")
    codes, scales = O.quantize_pages_bulk(g["values"], g["center"], "half_even")
    assert np.array_equal(scales.view(np.uint16), g["scale"].view(np.uint16))
    assert np.array_equal(codes, g["codes"])
    # The oracle's own centre agrees with the reference's FP32 mean to 1 ulp.
    _, center, _ = O.quantize_page_gauge(g["values"])
    diff = np.abs(center.view(np.uint16).astype(np.int32) - g["center"].view(np.uint16).astype(np.int32))
    assert diff.max() <= 1
    # Reconstruction identity of the reference test (test_flashinfer_page_affine_int8.py:36-47).
    recon = (codes.astype(np.float32) * scales.astype(np.float32)[:, None, :, None]).astype(np.float16)
    assert np.array_equal(recon.view(np.uint16), g["reconstructed"].view(np.uint16))


def test_half_away_and_half_even_differ_only_on_ties():
    g = np.load(GOLDEN / "quantize_page_gauge.npz")
    a, sa = O.quantize_pages_bulk(g["values"], g["center"], "half_away")
    e, se = O.quantize_pages_bulk(g["values"], g["center"], "half_even")
    assert np.array_equal(sa, se)
    q = (g["values"].astype(np.float32) - g["center"].astype(np.float32)[None, None]) / \
        sa.astype(np.float32)[:, None, :, None]
    # floor(|q| + 0.5) in float32 also rounds up when |q| + 0.5 is not
    # representable just below an integer, so "near ties" count as ties.
    frac = np.abs(np.abs(q) - np.trunc(np.abs(q)) - 0.5)
    near_tie = frac <= np.abs(q) * 2.0**-22
    differ = a != e
    assert np.all(near_tie[differ])
    assert np.all(np.abs(a.astype(np.int32) - e.astype(np.int32)) <= 1)


def test_rope_matches_torch_fp16_expression_bitwise():
    g = np.load(GOLDEN / "rope.npz")
    for i, p in enumerate(g["positions"]):
        rq = O.rope_fp16(g["q"], g["cos"][p], g["sin"][p])
        rk = O.rope_fp16(g["k"], g["cos"][p], g["sin"][p])
        assert np.array_equal(rq.view(np.uint16), g["expected_q"][i].view(np.uint16))
        assert np.array_equal(rk.view(np.uint16), g["expected_k"][i].view(np.uint16))


def test_completed_page_scale_algebra_pin():
    g = np.load(GOLDEN / "scale_pin.npz")
    _, scales = O.quantize_pages_bulk(g["key"], g["center"], "half_away")
    assert np.array_equal(scales.view(np.uint16), g["expected_scale"].view(np.uint16))


@pytest.mark.parametrize("tail_tokens", [1, 15, 16, 17, 241, 255, 256])
def test_tail_merge_oracle_matches_reference_formula(tail_tokens):
    g = np.load(GOLDEN / "tail_merge.npz")
    p = f"t{tail_tokens}_"
    out, lse = O.exact_tail_merge_center(
        g["query"][0], g["exact_k"], g["exact_v"], g[p + "indices"], tail_tokens,
        g[p + "old_out"][0], g[p + "old_lse"][0], g["value_center"], 128 ** -0.5)
    np.testing.assert_allclose(out, g[p + "expected_out"][0], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(lse, g[p + "expected_lse"][0], atol=2e-5, rtol=1e-6)


def _state(B, exact_ppr, code_ppr, hkv=8):
    return O.GaugeState(
        exact_k=np.zeros((B * exact_ppr, 16, hkv, 128), np.float16),
        exact_v=np.zeros((B * exact_ppr, 16, hkv, 128), np.float16),
        codes_k=np.zeros((B * code_ppr, 16, hkv, 128), np.int8),
        codes_v=np.zeros((B * code_ppr, 16, hkv, 128), np.int8),
        scales_k=np.zeros((B * code_ppr, hkv), np.float16),
        scales_v=np.zeros((B * code_ppr, hkv), np.float16),
    )


def test_append_oracle_ring_reuse_and_reconstruction():
    """Scenario of tests/test_page_gauge_append_extension.py:218-279 on the oracle."""
    rng = np.random.default_rng(73)
    pages, ring = 4, 2
    q = rng.standard_normal((1, 32, 128)).astype(np.float16)
    keys = rng.standard_normal((pages * 16, 1, 8, 128)).astype(np.float16)
    values = rng.standard_normal((pages * 16, 1, 8, 128)).astype(np.float16)
    cos = np.ones(128, np.float16)
    sin = np.zeros(128, np.float16)
    kc = (rng.standard_normal((8, 128)) * 0.1).astype(np.float16)
    vc = (rng.standard_normal((8, 128)) * 0.1).astype(np.float16)
    st = _state(1, ring, pages)
    for pos in range(pages * 16):
        rq = O.rope_append_page_gauge(st, q, keys[pos], values[pos], cos, sin, kc, vc, 0, pos)
    assert np.array_equal(rq, q)
    recon = st.codes_k.astype(np.float32) * st.scales_k.astype(np.float32)[:, None, :, None] + kc.astype(np.float32)
    ref = keys[:, 0].reshape(pages, 16, 8, 128).astype(np.float32)
    assert np.linalg.norm(recon - ref) / np.linalg.norm(ref) < 0.02
    for lp in (2, 3):
        np.testing.assert_allclose(st.exact_k[lp % ring].astype(np.float32) + kc.astype(np.float32),
                                   ref[lp], atol=2e-3, rtol=0)


def test_append_oracle_sink_slot_survives_wraps():
    """Scenario of tests/test_page_gauge_append_extension.py:282-349."""
    rng = np.random.default_rng(20260820)
    pages, tail, sink = 5, 2, 1
    q = rng.standard_normal((1, 32, 128)).astype(np.float16)
    keys = rng.standard_normal((pages * 16, 1, 8, 128)).astype(np.float16)
    values = rng.standard_normal((pages * 16, 1, 8, 128)).astype(np.float16)
    cos, sin = np.ones(128, np.float16), np.zeros(128, np.float16)
    kc = (rng.standard_normal((8, 128)) * 0.1).astype(np.float16)
    vc = (rng.standard_normal((8, 128)) * 0.1).astype(np.float16)
    st = _state(1, sink + tail, pages)
    for pos in range(pages * 16):
        O.rope_append_page_gauge(st, q, keys[pos], values[pos], cos, sin, kc, vc, sink, pos)
    ref_k = keys[:, 0].reshape(pages, 16, 8, 128).astype(np.float32)
    np.testing.assert_allclose(st.exact_k[0].astype(np.float32) + kc.astype(np.float32), ref_k[0], atol=2e-3, rtol=0)
    for lp in (3, 4):
        np.testing.assert_allclose(st.exact_k[sink + lp % tail].astype(np.float32) + kc.astype(np.float32),
                                   ref_k[lp], atol=2e-3, rtol=0)


def test_attention_oracle_segments_equal_dense_reconstruction():
    """Factorised decode over (old INT8, exact FP16) equals dense attention
    over the reconstructed cache (the identity the reference benchmark
    checks, scripts/benchmark_flashinfer_page_affine_int8.py:644-648)."""
    rng = np.random.default_rng(5)
    pages, tail = 20, 4
    vals_k = (rng.standard_normal((pages, 16, 8, 128)) * 0.35).astype(np.float16)
    vals_v = (rng.standard_normal((pages, 16, 8, 128)) * 0.35).astype(np.float16)
    q = rng.standard_normal((32, 128)).astype(np.float16)
    ck, center_k, sk = O.quantize_page_gauge(vals_k)
    cv, center_v, sv = O.quantize_page_gauge(vals_v)
    old = list(range(pages - tail))
    ex = list(range(pages - tail, pages))
    exact_k = (vals_k.astype(np.float32) - center_k.astype(np.float32)).astype(np.float16)
    exact_v = (vals_v.astype(np.float32) - center_v.astype(np.float32)).astype(np.float16)
    out, lse = O.page_gauge_decode(q, ck, cv, sk, sv, old, len(old) * 16, exact_k, exact_v, ex,
                                   len(ex) * 16, center_v, 128 ** -0.5)
    keys = np.concatenate([O.dequant_tokens(ck, sk, old, len(old) * 16),
                           O.gather_tokens(exact_k, ex, len(ex) * 16).astype(np.float64)])
    vals = np.concatenate([O.dequant_tokens(cv, sv, old, len(old) * 16),
                           O.gather_tokens(exact_v, ex, len(ex) * 16).astype(np.float64)])
    dense, dense_lse = O.attention_state(q, keys, vals, 128 ** -0.5)
    dense = dense + np.repeat(center_v.astype(np.float64), 4, axis=0)
    np.testing.assert_allclose(out, dense, atol=1e-12)
    np.testing.assert_allclose(lse, dense_lse, atol=1e-10)
    # c_K cancels: shifting every key by a per-channel constant leaves the
    # softmax unchanged up to the constant row offset.
    shifted, _ = O.attention_state(q, keys + center_k.astype(np.float64)[None], vals, 128 ** -0.5)
    np.testing.assert_allclose(shifted + np.repeat(center_v.astype(np.float64), 4, axis=0), dense, atol=1e-10)


def test_affine_group16_quantiser_bit_exact_against_reference():
    """quantize_pages (scripts/benchmark_flashinfer_page_affine_int8.py:234-253),
    run by the reference on CPU: random pages, a constant page (scale
    floor) and a page of exact half-step ties (half to even)."""
    g = np.load(GOLDEN / "quantize_affine_group16.npz")
    codes, bias, scale, recon = O.quantize_pages_affine(g["values"])
    np.testing.assert_array_equal(codes, g["codes"])
    np.testing.assert_array_equal(bias.view(np.uint16), g["bias"].view(np.uint16))
    np.testing.assert_array_equal(scale.view(np.uint16), g["scale"].view(np.uint16))
    np.testing.assert_array_equal(recon.view(np.uint16), g["reconstructed"].view(np.uint16))
    # The tie page really has ties: (x - min) / scale = k + 0.5 exactly.
    x = g["values"][2].astype(np.float32)
    assert np.any(np.mod(x / np.float32(0.125), 1) == 0.5)
    assert np.all(scale[1] == np.float16(2.0**-20))


def test_affine_tokens_match_the_reference_reconstruction():
    """The decode oracle's single-rounding rebuild fp16(z*s+b) equals the
    reference's fp32 product + add + fp16 cast except where the two roundings
    differ (at most one FP16 step)."""
    g = np.load(GOLDEN / "quantize_affine_group16.npz")
    ids = [0, 3, 1]
    got = O.affine_tokens(g["codes"], g["bias"], g["scale"], ids, 40)
    ref = g["reconstructed"][ids].reshape(-1, 8, 128)[:40].astype(np.float64)
    step = np.abs(ref) * 2.0 ** -10 + 2.0 ** -24
    assert np.all(np.abs(got - ref) <= step)
    assert np.mean(got == ref) > 0.99
