"""Property tests of the CPU oracle itself (the checker every parity test
relies on): the quantiser's scale rule, code range and reconstruction
bound, round-half-away versus half-even on ties, and the LSE merge being
the attention over the union of the merged token sets (split invariance),
in any grouping."""

from __future__ import annotations

import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from oracle import pagegauge_oracle as O  # noqa: E402


@settings(max_examples=60, deadline=None)
@given(st.integers(0, 2**31 - 1), st.integers(1, 4), st.integers(1, 3),
       st.floats(1e-3, 1e3), st.sampled_from(["half_away", "half_even"]))
def test_quantiser_scale_range_and_error_bound(seed, pages, hkv, spread, rounding):
    rng = np.random.default_rng(seed)
    vals = (rng.standard_normal((pages, 16, hkv, 128)) * spread).astype(np.float16)
    center = (rng.standard_normal((hkv, 128)) * spread).astype(np.float16)
    codes, scales = O.quantize_pages_bulk(vals, center, rounding)
    centred = vals.astype(np.float32) - center.astype(np.float32)[None, None]
    absmax = np.abs(centred).max(axis=(1, 3))
    # The scale rule, bit for bit.
    expect = np.maximum(absmax / np.float32(127), np.float32(2.0 ** -20)).astype(np.float16)
    assert np.array_equal(scales, expect)
    assert codes.dtype == np.int8 and np.abs(codes.astype(np.int32)).max() <= 127
    # Reconstruction within half a step (the FP16 scale rounds absmax/127 to
    # 11 bits, so the extreme code may clamp: allow that step's rounding).
    s = scales.astype(np.float32)[:, None, :, None]
    err = np.abs(centred - codes.astype(np.float32) * s)
    assert np.all(err <= 0.5 * s * (1 + 2.0 ** -9) + np.abs(centred) * 2.0 ** -10 + 1e-30)


def test_rounding_modes_differ_only_on_ties():
    q = np.array([-2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 0.49, -0.51, 3.7], np.float32)
    away = O.round_half_away(q)
    even = np.rint(q).astype(np.int32)
    assert away.tolist() == [-3, -2, -1, 1, 2, 3, 0, -1, 4]
    ties = np.abs(q - np.trunc(q)) == 0.5
    assert np.array_equal(away[~ties], even[~ties])


@settings(max_examples=60, deadline=None)
@given(st.integers(0, 2**31 - 1), st.lists(st.integers(0, 40), min_size=1, max_size=5))
def test_merge_of_splits_equals_attention_over_the_union(seed, sizes):
    rng = np.random.default_rng(seed)
    hkv, hq = 2, 8
    total = sum(sizes)
    q = rng.standard_normal((hq, 128)).astype(np.float16)
    k = rng.standard_normal((max(total, 1), hkv, 128)).astype(np.float16)[:total]
    v = rng.standard_normal((max(total, 1), hkv, 128)).astype(np.float16)[:total]
    sm = O.sm_scale_default()
    whole_o, whole_l = O.attention_state(q, k, v, sm)
    parts, at = [], 0
    for n in sizes:
        parts.append(O.attention_state(q, k[at:at + n], v[at:at + n], sm))
        at += n
    merged_o, merged_l = O.merge_states(parts)
    if total == 0:
        assert np.all(np.isneginf(merged_l)) and np.all(merged_o == 0)
        return
    assert np.allclose(merged_o, whole_o, rtol=1e-10, atol=1e-12)
    assert np.allclose(merged_l, whole_l, rtol=1e-12, atol=1e-12)
    # Any grouping of the partial states gives the same result.
    if len(parts) > 2:
        left = O.merge_states(parts[:2])
        regrouped = O.merge_states([left] + parts[2:])
        assert np.allclose(regrouped[0], whole_o, rtol=1e-10, atol=1e-12)
