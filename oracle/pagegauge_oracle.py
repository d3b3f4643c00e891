"""Numpy restatement of the PageGauge INT8 page-affine decode path.

TEST INFRASTRUCTURE ONLY -- the product never imports this module.

Each function names the reference code (path inside ahmed123hds/PageGauge)
whose arithmetic it restates.  Integer/byte outputs (codes, scales, ring
contents, rotated queries) are meant to be compared bit-exactly; attention
outputs are computed in float64 and compared within the tolerance the
caller states.

FP16 arithmetic note: a single IEEE binary16 multiply or add is emulated as
``float32 op`` followed by a round-to-nearest-even cast to float16.  The
product of two binary16 values is exact in float32, and binary32 carries
2*11+2 significand bits, so the double rounding of a sum is innocuous: the
result equals the correctly rounded binary16 operation.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

PAGE = 16
DIM = 128
LOG2E = 1.4426950408889634
SCALE_FLOOR = np.float32(2.0**-20)


# --------------------------------------------------------------------- RoPE
def f16_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.float32) * b.astype(np.float32)).astype(np.float16)


def f16_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16)


def rope_fp16(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """HF rotate-half RoPE with every product and the sum rounded to FP16.

    tests/page_gauge_append_extension.cu:148-180 (rotate_element), pinned
    bitwise to ``q*cos + cat(-q[64:], q[:64])*sin`` in torch FP16 by
    tests/test_page_gauge_append_extension.py:75-92.
    """
    x = np.asarray(x, dtype=np.float16)
    partner = np.concatenate([-x[..., DIM // 2 :], x[..., : DIM // 2]], axis=-1)
    return f16_add(f16_mul(x, cos), f16_mul(partner, sin))


# ------------------------------------------------------------ quantisation
def page_scale(absmax: np.ndarray) -> np.ndarray:
    """fp16(max(absmax / 127, 2^-20)) with IEEE float32 division.

    tests/page_gauge_append_extension.cu:346-351; the same rule in
    scripts/benchmark_page_gauge_overheads.py:55-64 and its torch pin
    tests/test_page_gauge_overheads.py:54-63.
    """
    q = np.asarray(absmax, dtype=np.float32) / np.float32(127.0)
    return np.maximum(q, SCALE_FLOOR).astype(np.float16)


def round_half_away(q: np.ndarray) -> np.ndarray:
    """sign(q) * floor(|q| + 0.5) in float32 (.cu:372-377; overheads :65-73)."""
    q = np.asarray(q, dtype=np.float32)
    pos = np.floor(q + np.float32(0.5))
    neg = -np.floor(-q + np.float32(0.5))
    return np.where(q >= 0, pos, neg).astype(np.int32)


def quantize_codes(values: np.ndarray, scale: np.ndarray, rounding: str) -> np.ndarray:
    """Codes = clamp(round(values / scale), -127, 127) as int8.

    values float32 (already centred), scale broadcastable float16.
    rounding: "half_away" (CUDA/Triton kernels) or "half_even" (torch.round in
    quantize_page_gauge, scripts/benchmark_flashinfer_page_affine_int8.py:266-270).
    """
    q = np.asarray(values, dtype=np.float32) / np.asarray(scale).astype(np.float32)
    if rounding == "half_away":
        z = round_half_away(q)
    elif rounding == "half_even":
        z = np.rint(q).astype(np.int32)
    else:
        raise ValueError(rounding)
    return np.clip(z, -127, 127).astype(np.int8)


def quantize_pages_bulk(
    values: np.ndarray, center: np.ndarray, rounding: str = "half_away"
) -> tuple[np.ndarray, np.ndarray]:
    """Completed-page quantiser over [pages, 16, Hkv, 128] FP16 pages.

    scripts/benchmark_page_gauge_overheads.py:51-83 (fp32 centring, not
    rounded to FP16; one scale per (page, head)).  ``center`` is [Hkv,128]
    or [pages, Hkv, 128] (per-page centre rows).
    Returns (codes int8 [pages,16,Hkv,128], scales fp16 [pages,Hkv]).
    """
    v = values.astype(np.float32)
    c = np.asarray(center, dtype=np.float16).astype(np.float32)
    if c.ndim == 2:
        c = c[None, None]
    else:
        c = c[:, None]
    centred = v - c
    absmax = np.abs(centred).max(axis=(1, 3))  # [pages, Hkv]
    scales = page_scale(absmax)
    codes = quantize_codes(centred, scales[:, None, :, None], rounding)
    return codes, scales


def quantize_page_gauge(values: np.ndarray):
    """Restatement of quantize_page_gauge
    (scripts/benchmark_flashinfer_page_affine_int8.py:256-278): centre =
    fp16(mean over all pages and tokens), one scale per (page, head),
    round-half-to-even codes.  The mean is taken in float64 and rounded to
    float32 then float16; the reference's float32 reduction order can differ
    in the last float32 bit, so callers that need bit-exact codes pass the
    reference's own centre to ``quantize_pages_bulk``.
    """
    center = values.astype(np.float64).mean(axis=(0, 1)).astype(np.float32).astype(np.float16)
    codes, scales = quantize_pages_bulk(values, center, "half_even")
    return codes, center, scales


def quantize_pages_affine(values: np.ndarray):
    """The reference's alternative "affine_group16" representation,
    quantize_pages (scripts/benchmark_flashinfer_page_affine_int8.py:234-253):
    per (page, head, 16-dim group) over the group's 16 tokens x 16 dims in
    float32, scale = fp16(max((max - min) / 255, 2^-20)), mn = fp16(min),
    u = clamp(rint((x - mn) / scale), 0, 255) (half to even), code = u - 128,
    bias = fp16(mn + fp16(128 * scale)), reconstructed = fp16(fp32(code *
    scale) + bias).  Returns (codes int8 [P,16,H,128], bias fp16 [P,H,8],
    scale fp16 [P,H,8], reconstructed fp16 [P,16,H,128])."""
    v = np.asarray(values, np.float16)
    P, T, H, D = v.shape
    G = D // 16
    x = v.astype(np.float32).transpose(0, 2, 1, 3).reshape(P, H, T, G, 16)
    mn = x.min(axis=(2, 4), keepdims=True)
    mx = x.max(axis=(2, 4), keepdims=True)
    scale = np.maximum((mx - mn) / np.float32(255.0), SCALE_FLOOR).astype(np.float16)
    mn16 = mn.astype(np.float16)
    s32 = scale.astype(np.float32)
    u = np.clip(np.rint((x - mn16.astype(np.float32)) / s32), 0, 255)
    signed = (u - 128).astype(np.int8)
    b128 = (np.float32(128.0) * s32).astype(np.float16)
    bias = (mn16.astype(np.float32) + b128.astype(np.float32)).astype(np.float16)
    recon = (signed.astype(np.float32) * s32 + bias.astype(np.float32)).astype(np.float16)
    codes = signed.reshape(P, H, T, D).transpose(0, 2, 1, 3)
    recon = recon.reshape(P, H, T, D).transpose(0, 2, 1, 3)
    return (np.ascontiguousarray(codes), bias.reshape(P, H, G), scale.reshape(P, H, G),
            np.ascontiguousarray(recon))


def affine_tokens(codes, bias, scale, ids, n_tokens):
    """Old-page tokens of the affine_group16 representation as the reference's
    FA2 variant rebuilds them (patch compute_qk affine branch: code -> half,
    one half2 FMA with the group's scale and bias): fp16(z * s + b), rounded
    once.  Returns float64 [n_tokens, Hkv, 128]."""
    ids = np.asarray(ids, dtype=np.int64)
    if ids.size == 0:
        return np.zeros((0,) + codes.shape[2:])
    z = codes[ids].astype(np.float64)                                    # [n,16,H,128]
    s = np.repeat(scale[ids].astype(np.float64), 16, axis=-1)[:, None]  # [n,1,H,128]
    b = np.repeat(bias[ids].astype(np.float64), 16, axis=-1)[:, None]
    x = (z * s + b).astype(np.float16).astype(np.float64)
    return x.reshape((-1,) + codes.shape[2:])[:n_tokens]


def affine_decode(q, codes_k, codes_v, k_bias, k_scale, v_bias, v_scale, old_ids, old_tokens,
                  exact_k=None, exact_v=None, exact_ids=(), exact_tokens=0, sm_scale=None):
    """affine_group16 decode of one request (scripts/benchmark_flashinfer_page_affine_int8.py:
    567-602): old pages rebuilt per group, optional FP16 exact segment merged
    by LSE; no centres.  Returns (output float64 [Hq,128], lse base 2)."""
    sm_scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(DIM)
    hq = q.shape[0]
    states = []
    if old_tokens:
        states.append(attention_state(q, affine_tokens(codes_k, k_bias, k_scale, old_ids, old_tokens),
                                      affine_tokens(codes_v, v_bias, v_scale, old_ids, old_tokens),
                                      sm_scale))
    if exact_tokens:
        states.append(attention_state(q, gather_tokens(exact_k, exact_ids, exact_tokens).astype(np.float64),
                                      gather_tokens(exact_v, exact_ids, exact_tokens).astype(np.float64),
                                      sm_scale))
    if not states:
        return np.zeros((hq, DIM)), np.full(hq, -np.inf)
    return merge_states(states)


# ----------------------------------------------------------------- append
@dataclass
class GaugeState:
    """Per-layer PageGauge storage, request-major (GaugeCache,
    scripts/benchmark_page_gauge_transformer.py:321-380)."""

    exact_k: np.ndarray  # fp16 [B*exact_ppr, 16, Hkv, 128]
    exact_v: np.ndarray
    codes_k: np.ndarray  # int8 [B*code_ppr, 16, Hkv, 128]
    codes_v: np.ndarray
    scales_k: np.ndarray  # fp16 [B*code_ppr, Hkv]
    scales_v: np.ndarray


def rope_append_page_gauge(
    state: GaugeState,
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    cos: np.ndarray,
    sin: np.ndarray,
    key_center: np.ndarray,
    value_center: np.ndarray,
    exact_sink_pages: int,
    position: int,
) -> np.ndarray:
    """One fused append step; mutates ``state`` and returns the rotated q.

    tests/page_gauge_append_extension.cu:244-383: RoPE q and k, centre K/V in
    float32 and round to FP16 into ring slot ``sink + page % tail`` (or the
    prefix slot), and on token 15 finalise the page: abs-max of the FP16
    ring page, scale, half-away codes.
    """
    B, hq, _ = q.shape
    hkv = k.shape[1]
    exact_ppr = state.exact_k.shape[0] // B
    code_ppr = state.codes_k.shape[0] // B
    page, token = divmod(position, PAGE)
    tail = exact_ppr - exact_sink_pages
    local = page if page < exact_sink_pages else exact_sink_pages + page % tail
    kc = np.broadcast_to(np.asarray(key_center, np.float16), (B, hkv, DIM))
    vc = np.broadcast_to(np.asarray(value_center, np.float16), (B, hkv, DIM))
    rq = rope_fp16(q, cos, sin)
    rk = rope_fp16(k, cos, sin)
    ck = (rk.astype(np.float32) - kc.astype(np.float32)).astype(np.float16)
    cv = (np.asarray(v, np.float16).astype(np.float32) - vc.astype(np.float32)).astype(np.float16)
    for r in range(B):
        ring = r * exact_ppr + local
        state.exact_k[ring, token] = ck[r]
        state.exact_v[ring, token] = cv[r]
        if token != PAGE - 1:
            continue
        cp = r * code_ppr + page
        for ring_arr, code_arr, scale_arr in (
            (state.exact_k, state.codes_k, state.scales_k),
            (state.exact_v, state.codes_v, state.scales_v),
        ):
            pg = ring_arr[ring].astype(np.float32)  # [16, Hkv, 128]
            sc = page_scale(np.abs(pg).max(axis=(0, 2)))  # [Hkv]
            scale_arr[cp] = sc
            code_arr[cp] = quantize_codes(pg, sc[None, :, None], "half_away")
    return rq


def rope_append_page_gauge_batched(
    state: GaugeState,
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    cos_table: np.ndarray,
    sin_table: np.ndarray,
    key_center: np.ndarray,
    value_center: np.ndarray,
    exact_sink_pages: int,
    positions,
) -> np.ndarray:
    """``rope_append_page_gauge`` with one position per request: request r
    runs the single-request step at ``positions[r]`` on its own slice of the
    request-major storage.  Per-request page ids and in-page offsets are the
    reference's Triton append_finalize_page_gauge
    (scripts/benchmark_page_gauge_overheads.py:113-205); the arithmetic per
    request is the extension kernel's (.cu:244-383)."""
    B = q.shape[0]
    exact_ppr = state.exact_k.shape[0] // B
    code_ppr = state.codes_k.shape[0] // B
    shared = np.asarray(key_center).ndim == 2
    out = np.empty_like(np.asarray(q, np.float16))
    for r, pos in enumerate(positions):
        e, c = slice(r * exact_ppr, (r + 1) * exact_ppr), slice(r * code_ppr, (r + 1) * code_ppr)
        sub = GaugeState(state.exact_k[e], state.exact_v[e], state.codes_k[c], state.codes_v[c],
                         state.scales_k[c], state.scales_v[c])
        kc = key_center if shared else key_center[r:r + 1]
        vc = value_center if shared else value_center[r:r + 1]
        out[r] = rope_append_page_gauge(sub, q[r:r + 1], k[r:r + 1], v[r:r + 1], cos_table[pos],
                                        sin_table[pos], kc, vc, exact_sink_pages, int(pos))[0]
    return out


def rope_append_fp16(
    key_pages: np.ndarray,
    value_pages: np.ndarray,
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    cos: np.ndarray,
    sin: np.ndarray,
    position: int,
) -> np.ndarray:
    """FP16 comparator: RoPE(q), RoPE(k) and raw v into page
    ``r*ppr + position//16`` (tests/page_gauge_append_extension.cu:182-242)."""
    B = q.shape[0]
    ppr = key_pages.shape[0] // B
    page, token = divmod(position, PAGE)
    rq = rope_fp16(q, cos, sin)
    rk = rope_fp16(k, cos, sin)
    for r in range(B):
        key_pages[r * ppr + page, token] = rk[r]
        value_pages[r * ppr + page, token] = v[r]
    return rq


def rope_append_fp16_batched(key_pages, value_pages, q, k, v, cos_table, sin_table, positions):
    """FP16 comparator with one position per request (request r writes page
    ``r*ppr + positions[r]//16``)."""
    B = q.shape[0]
    ppr = key_pages.shape[0] // B
    out = np.empty_like(np.asarray(q, np.float16))
    for r, pos in enumerate(positions):
        sl = slice(r * ppr, (r + 1) * ppr)
        out[r] = rope_append_fp16(key_pages[sl], value_pages[sl], q[r:r + 1], k[r:r + 1],
                                  v[r:r + 1], cos_table[pos], sin_table[pos], int(pos))[0]
    return out


# --------------------------------------------------------------- attention
def gather_tokens(pages: np.ndarray, ids, n_tokens: int) -> np.ndarray:
    """Concatenate the pages ``ids`` of a [P,16,Hkv,128] cache and keep the
    first ``n_tokens`` rows -> [n_tokens, Hkv, 128]."""
    if len(ids) == 0:
        return np.zeros((0,) + pages.shape[2:], dtype=pages.dtype)
    return pages[np.asarray(ids, dtype=np.int64)].reshape((-1,) + pages.shape[2:])[:n_tokens]


def dequant_tokens(codes, scales, ids, n_tokens):
    """Old-page reconstruction s * Z without the centre (centred domain),
    scripts/benchmark_flashinfer_page_affine_int8.py:274-276."""
    ids = np.asarray(ids, dtype=np.int64)
    z = gather_tokens(codes, ids, n_tokens).astype(np.float64)
    s = np.repeat(scales[ids].astype(np.float64), PAGE, axis=0)[:n_tokens]  # [T, Hkv]
    return z * s[:, :, None]


def attention_state(q: np.ndarray, keys: np.ndarray, values: np.ndarray, sm_scale: float):
    """Exact decode attention of one request over [T, Hkv, 128] keys/values.

    Returns (O float64 [Hq,128] normalised, lse base 2 [Hq]); empty T gives
    (0, -inf).  Scores are in log2 units (sm_scale*log2 e), the convention
    of the tail oracle tests/test_page_gauge_append_extension.py:628-657.
    """
    hq = q.shape[0]
    hkv = keys.shape[1]
    group = hq // hkv
    T = keys.shape[0]
    if T == 0:
        return np.zeros((hq, DIM)), np.full(hq, -np.inf)
    kv_for_q = np.arange(hq) // group
    qf = q.astype(np.float64)
    k = keys.astype(np.float64)[:, kv_for_q]  # [T, Hq, D]
    v = values.astype(np.float64)[:, kv_for_q]
    s = np.einsum("qd,tqd->qt", qf, k) * (sm_scale * LOG2E)
    m = s.max(axis=1, keepdims=True)
    w = np.exp2(s - m)
    den = w.sum(axis=1)
    out = np.einsum("qt,tqd->qd", w, v) / den[:, None]
    return out, m[:, 0] + np.log2(den)


def merge_states(states):
    """LSE merge of normalised partial states (flashinfer merge_state
    semantics, base 2): O = sum 2^(lse_i-m) O_i / sum 2^(lse_i-m)."""
    outs = np.stack([o for o, _ in states])
    lses = np.stack([l for _, l in states])
    m = lses.max(axis=0)
    finite = np.isfinite(m)
    safe = np.where(finite, m, 0.0)
    w = np.where(np.isfinite(lses), np.exp2(lses - safe[None]), 0.0)
    den = w.sum(axis=0)
    out = np.where(den[:, None] > 0, (w[:, :, None] * outs).sum(axis=0) / np.maximum(den, 1e-300)[:, None], 0.0)
    lse = np.where(den > 0, safe + np.log2(np.maximum(den, 1e-300)), -np.inf)
    return out, lse


def page_gauge_decode(
    q: np.ndarray,
    codes_k, codes_v, scales_k, scales_v, old_ids, old_tokens,
    exact_k, exact_v, exact_ids, exact_tokens,
    value_center, sm_scale: float,
):
    """Full PageGauge decode attention for one request.

    Old INT8 segment (centred reconstruction s*Z) and exact centred FP16
    segment are two partial states merged by LSE, then c_V is added:
    scripts/benchmark_flashinfer_page_affine_int8.py:581-602 and
    scripts/benchmark_page_gauge_transformer.py:2261-2308.
    Returns (output float64 [Hq,128], lse base 2 of the centred attention).
    """
    hq = q.shape[0]
    hkv = codes_k.shape[2] if codes_k is not None else exact_k.shape[2]
    states = []
    if old_tokens:
        ko = dequant_tokens(codes_k, scales_k, old_ids, old_tokens)
        vo = dequant_tokens(codes_v, scales_v, old_ids, old_tokens)
        states.append(attention_state(q, ko, vo, sm_scale))
    if exact_tokens:
        ke = gather_tokens(exact_k, exact_ids, exact_tokens).astype(np.float64)
        ve = gather_tokens(exact_v, exact_ids, exact_tokens).astype(np.float64)
        states.append(attention_state(q, ke, ve, sm_scale))
    out, lse = merge_states(states) if states else (np.zeros((hq, DIM)), np.full(hq, -np.inf))
    if value_center is not None:
        group = hq // hkv
        out = out + np.repeat(np.asarray(value_center, np.float64), group, axis=0)
    return out, lse


def exact_tail_merge_center(q, exact_k, exact_v, ids, tail_tokens, old_out, old_lse, value_center, sm_scale):
    """Reference oracle of exact_tail_merge_center for one request
    (tests/test_page_gauge_append_extension.py:628-657)."""
    ke = gather_tokens(exact_k, ids, tail_tokens).astype(np.float64)
    ve = gather_tokens(exact_v, ids, tail_tokens).astype(np.float64)
    tail = attention_state(q, ke, ve, sm_scale)
    out, lse = merge_states([(np.asarray(old_out, np.float64), np.asarray(old_lse, np.float64)), tail])
    hq = q.shape[0]
    group = hq // exact_k.shape[2]
    return out + np.repeat(np.asarray(value_center, np.float64), group, axis=0), lse


def merge_state_in_place(va, sa, vb, sb):
    """flashinfer.merge_state_in_place restated on [rows,128]/[rows]."""
    out, lse = merge_states([(va.astype(np.float64), sa.astype(np.float64)),
                             (vb.astype(np.float64), sb.astype(np.float64))])
    return out, lse


# -------------------------------------------------------------- metrics
def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


def sm_scale_default() -> float:
    return 1.0 / math.sqrt(DIM)
