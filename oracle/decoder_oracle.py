"""CPU restatement of the PageGauge decoder (test infrastructure only: the
GPU decoder's parity tests, smoke() and bench.py's CPU baseline may call it;
the product never does).

The layer body follows the reference decoder
(scripts/benchmark_page_gauge_transformer.py:2754-2804: packed qkv, the
fused append, segmented PageGauge attention + c_V, o_proj, residual,
RMSNorm, packed gate/up, SiLU * up, down_proj) and transformers'
MistralForCausalLM for the dense prefill.  With ``round16=True`` every
tensor the GPU stores in FP16 is rounded to FP16 at the same points (GEMM
outputs, norm outputs, residual sums, activations), accumulations are FP32
and attention is float64; with ``round16=False`` the dense forward is plain
FP32, which is what the tests pin against transformers' model.

Weights are numpy arrays laid out as the product packs them: per layer
``attn_norm [H]``, ``qkv [(hq+2hkv)*128, H]`` (q | k | v rows), ``o [H, hq*128]``,
``mlp_norm [H]``, ``gate_up [2F, H]`` (gate | up rows), ``down [H, F]``;
plus ``embed [V, H]``, ``final_norm [H]``, ``lm_head [V, H]``.
"""

from __future__ import annotations

import numpy as np

from . import pagegauge_oracle as O

PAGE = 16
DIM = 128


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def linear(x, w, round16=True):
    y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    return _f16(y) if round16 else y


def rms_norm(x, w, eps, round16=True):
    """transformers MistralRMSNorm: FP32 x * rsqrt(mean(x^2) + eps), cast to
    the input dtype, times the weight."""
    xf = np.asarray(x, np.float32)
    n = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + np.float32(eps))
    if not round16:
        return np.asarray(w, np.float32) * n
    return _f16(np.asarray(w, np.float32) * _f16(n).astype(np.float32))


def silu_mul(gu, features, round16=True):
    g = np.asarray(gu[..., :features], np.float32)
    u = np.asarray(gu[..., features:], np.float32)
    s = g / (np.float32(1) + np.exp(-g))
    if not round16:
        return s * u
    return _f16(_f16(s).astype(np.float32) * u)


def add(a, b, round16=True):
    y = np.asarray(a, np.float32) + np.asarray(b, np.float32)
    return _f16(y) if round16 else y


def rope(x, cos, sin, round16=True):
    """HF rotate-half RoPE; per-token tables [T, 128] broadcast over heads."""
    if round16:
        return O.rope_fp16(x, cos[:, None, :], sin[:, None, :])
    xf = np.asarray(x, np.float32)
    partner = np.concatenate([-xf[..., DIM // 2:], xf[..., :DIM // 2]], axis=-1)
    return xf * np.asarray(cos, np.float32)[:, None, :] + partner * np.asarray(sin, np.float32)[:, None, :]


def rope_tables(positions, theta):
    """transformers' rotary tables: FP32 angles t * theta^(-2i/128),
    cat(freqs, freqs); returned in FP32 (round16=False) and FP16."""
    inv = 1.0 / (theta ** (np.arange(0, DIM, 2, dtype=np.int64).astype(np.float32) / DIM))
    t = np.arange(positions, dtype=np.float32)
    emb = np.outer(t, inv.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([emb, emb], axis=-1)
    return np.cos(emb), np.sin(emb)


def causal_attention(q, k, v, scale):
    """q [T, Hq, D], k/v [T, Hkv, D]; query head i reads KV head i // group;
    float64 softmax."""
    T, hq, _ = q.shape
    group = hq // k.shape[1]
    out = np.empty((T, hq, DIM), np.float64)
    mask = np.triu(np.ones((T, T), bool), 1)
    for h in range(hq):
        s = (np.asarray(q[:, h], np.float64) @ np.asarray(k[:, h // group], np.float64).T) * scale
        s[mask] = -np.inf
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[:, h] = p @ np.asarray(v[:, h // group], np.float64)
    return out


def dense_forward(w, cfg, tokens, reduce=None, round16=True, rope_cache=None):
    """Prefill of one request: returns (last-position logits [V_l] FP32, per
    layer post-RoPE keys and values [T, hkv, 128]).  ``reduce`` sums partial
    o/down outputs across tensor-parallel ranks (identity by default)."""
    reduce = reduce or (lambda x: x)
    T = len(tokens)
    hq, hkv = cfg["hq"], cfg["hkv"]
    cos32, sin32 = rope_cache if rope_cache is not None else rope_tables(T, cfg["theta"])
    cos, sin = (_f16(cos32[:T]), _f16(sin32[:T])) if round16 else (cos32[:T], sin32[:T])
    h = np.asarray(w["embed"][tokens], np.float16 if round16 else np.float32)
    kvs = []
    for lw in w["layers"]:
        x = rms_norm(h, lw["attn_norm"], cfg["eps"], round16)
        qkv = linear(x, lw["qkv"], round16)
        q = qkv[:, :hq * DIM].reshape(T, hq, DIM)
        k = qkv[:, hq * DIM:(hq + hkv) * DIM].reshape(T, hkv, DIM)
        v = qkv[:, (hq + hkv) * DIM:].reshape(T, hkv, DIM)
        q, k = rope(q, cos, sin, round16), rope(k, cos, sin, round16)
        kvs.append((k, v))
        att = causal_attention(q, k, v, DIM ** -0.5).reshape(T, hq * DIM)
        att = _f16(att) if round16 else att.astype(np.float32)
        o = reduce(linear(att, lw["o"], False))
        h = add(h, _f16(o) if round16 else o, round16)
        x = rms_norm(h, lw["mlp_norm"], cfg["eps"], round16)
        gu = linear(x, lw["gate_up"], round16)
        act = silu_mul(gu, gu.shape[-1] // 2, round16)
        d = reduce(linear(act, lw["down"], False))
        h = add(h, _f16(d) if round16 else d, round16)
    x = rms_norm(h[-1:], w["final_norm"], cfg["eps"], round16)
    return linear(x, w["lm_head"], round16)[0].astype(np.float32), kvs


def page_tables(positions, capacity_pages, ring_pages=16, sink_pages=0, suffix_pages=0,
                initial_pages=None):
    """Old/exact page ids per request for a step appending at positions[r]
    (page_gauge_logical_partition and exact_physical_page_index,
    benchmark_page_gauge_transformer.py:460-599): exact pages are the first
    sink_pages, the suffix_pages that ended an ``initial_pages`` prompt, and
    the current page with the ring_pages - 1 before it; the exact storage of
    a request is sink, suffix, then a ring slot ``fixed + page % ring``."""
    fixed = sink_pages + suffix_pages
    storage = fixed + ring_pages
    sbeg = initial_pages - suffix_pages if suffix_pages else None
    tables = []
    for r, p in enumerate(positions):
        cur = p // PAGE
        tail0 = max(0, cur - ring_pages + 1)
        old, exact = [], []
        for lp in range(cur + 1):
            if lp < sink_pages:
                exact.append(r * storage + lp)
            elif sbeg is not None and sbeg <= lp < initial_pages:
                exact.append(r * storage + sink_pages + lp - sbeg)
            elif lp >= tail0:
                exact.append(r * storage + fixed + lp % ring_pages)
            else:
                old.append(r * capacity_pages + lp)
        tables.append((old, exact, len(old) * PAGE, p + 1 - len(old) * PAGE))
    return tables


def decode_step(w, cfg, caches, tokens, positions, capacity_pages, ring_pages=16, sink_pages=0,
                suffix_pages=0, initial_pages=None):
    """One greedy decode step of the batch from the page-gauge caches
    (``caches[l]`` = dict with GaugeState ``state`` and FP16 ``key_center`` /
    ``value_center`` [B, hkv, 128]); mutates the caches with the fused append
    and returns the logits [B, V_l] FP32."""
    hq, hkv = cfg["hq"], cfg["hkv"]
    B = len(tokens)
    cos32, sin32 = cfg["rope"]
    cos, sin = _f16(cos32), _f16(sin32)
    h = np.asarray(w["embed"][np.asarray(tokens)], np.float16)
    tables = page_tables(positions, capacity_pages, ring_pages, sink_pages, suffix_pages,
                         initial_pages)
    for lw, c in zip(w["layers"], caches):
        x = rms_norm(h, lw["attn_norm"], cfg["eps"])
        qkv = linear(x, lw["qkv"])
        q = qkv[:, :hq * DIM].reshape(B, hq, DIM)
        k = qkv[:, hq * DIM:(hq + hkv) * DIM].reshape(B, hkv, DIM)
        v = qkv[:, (hq + hkv) * DIM:].reshape(B, hkv, DIM)
        st = c["state"]
        rq = O.rope_append_page_gauge_batched(st, q, k, v, cos, sin, c["key_center"],
                                              c["value_center"], sink_pages + suffix_pages,
                                              positions)
        att = np.empty((B, hq, DIM), np.float16)
        for r in range(B):
            old, exact, old_tok, ex_tok = tables[r]
            out, _ = O.page_gauge_decode(rq[r], st.codes_k, st.codes_v, st.scales_k, st.scales_v,
                                         old, old_tok, st.exact_k, st.exact_v, exact, ex_tok,
                                         c["value_center"][r], DIM ** -0.5)
            att[r] = _f16(out)
        h = add(h, linear(att.reshape(B, -1), lw["o"]))
        x = rms_norm(h, lw["mlp_norm"], cfg["eps"])
        gu = linear(x, lw["gate_up"])
        h = add(h, linear(silu_mul(gu, gu.shape[-1] // 2), lw["down"]))
    x = rms_norm(h, w["final_norm"], cfg["eps"])
    return linear(x, w["lm_head"]).astype(np.float32)
