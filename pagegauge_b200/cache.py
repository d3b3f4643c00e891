"""PageGauge cache containers and builders (GPU).

``GaugeCache`` mirrors scripts/benchmark_page_gauge_transformer.py:321-380:
exact centred FP16 storage (fixed prefix pages + tail ring), INT8 codes and
per-(page, head) FP16 scales for every logical page, per-(request, head)
key/value centres.  ``build_gauge_cache`` follows build_caches (:1156-1259):
centres are the FP32 channel mean of each request's initial prefix rounded
to FP16, every page is quantised with the completed-page quantiser, and the
exact pages hold FP16(FP32 value - FP32 centre).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .quantize import quantize_pages_into

PAGE = 16
DIM = 128


def rope_tables(positions: int, theta: float = 1.0e6, dim: int = DIM,
                device: torch.device | str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """HF-style rotary tables (fp32 angles, cat(freqs, freqs)) cast to FP16."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64, device=device).float() / dim))
    t = torch.arange(positions, dtype=torch.float32, device=device)
    emb = torch.outer(t, inv)
    emb = torch.cat((emb, emb), dim=-1)
    return emb.cos().half(), emb.sin().half()


def apply_rope_fp16(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, 128] fp16 with per-row cos/sin [T, 128]: the torch FP16
    expression x*cos + rotate_half(x)*sin (each op rounded to FP16)."""
    c = cos[:, None, :]
    s = sin[:, None, :]
    return x * c + torch.cat((-x[..., DIM // 2:], x[..., :DIM // 2]), dim=-1) * s


@dataclass
class GaugeCache:
    exact_key: torch.Tensor    # fp16 [B*(S+T), 16, Hkv, 128]
    exact_value: torch.Tensor
    key_codes: torch.Tensor    # int8 [total_pages, 16, Hkv, 128]
    value_codes: torch.Tensor
    key_scales: torch.Tensor   # fp16 [total_pages, Hkv]
    value_scales: torch.Tensor
    key_center: torch.Tensor   # fp16 [B, Hkv, 128]
    value_center: torch.Tensor
    exact_tail_pages: int
    exact_sink_pages: int = 0

    @property
    def output_center(self) -> torch.Tensor:
        group = 4
        return self.value_center.repeat_interleave(group, dim=1).contiguous()


@dataclass
class DecodeTables:
    """CSR page tables of the two segments (device int32) + host copies."""

    old_indptr: torch.Tensor
    old_indices: torch.Tensor
    exact_indptr: torch.Tensor
    exact_indices: torch.Tensor
    exact_last_page_len: torch.Tensor
    old_tokens: list[int]
    exact_tokens: list[int]


def build_gauge_cache(dense_k: torch.Tensor, dense_v: torch.Tensor, lengths: list[int],
                      exact_tail_pages: int = 16, exact_sink_pages: int = 0,
                      prefix_tokens: list[int] | None = None,
                      capacity_pages: int | None = None) -> tuple[GaugeCache, DecodeTables]:
    """Quantise a dense request-major cache [sum(pages), 16, Hkv, 128].

    Request r owns the ``ceil(lengths[r]/16)`` consecutive pages after those
    of requests < r.  The last ``exact_tail_pages`` logical pages (and the
    first ``exact_sink_pages``) are exact; the rest are read as INT8.
    Tokens past a request's length inside its last page are ignored by
    attention (masked by last_page_len).

    With ``capacity_pages`` the INT8 cache gives every request the same
    capacity (request r's logical page p at r*capacity_pages + p), the
    request-major layout of request_major_page_table
    (scripts/benchmark_page_gauge_transformer.py:383-407) that the append
    kernels address; otherwise the requests' pages are packed."""
    device = dense_k.device
    hkv = dense_k.shape[2]
    batch = len(lengths)
    pages = [math.ceil(n / PAGE) for n in lengths]
    starts = [sum(pages[:r]) for r in range(batch)]
    if dense_k.shape[0] < sum(pages):
        raise ValueError("dense cache is smaller than the requested lengths")
    if capacity_pages is not None:
        if capacity_pages < max(pages):
            raise ValueError("capacity_pages is smaller than the longest request")
        dst = [r * capacity_pages for r in range(batch)]
        code_pages = batch * capacity_pages
    else:
        dst, code_pages = starts, dense_k.shape[0]
    prefix_tokens = prefix_tokens or lengths
    key_center = torch.empty(batch, hkv, DIM, device=device, dtype=torch.float16)
    value_center = torch.empty_like(key_center)
    key_codes = torch.zeros(code_pages, PAGE, hkv, DIM, device=device, dtype=torch.int8)
    value_codes = torch.zeros_like(key_codes)
    key_scales = torch.zeros(code_pages, hkv, device=device, dtype=torch.float16)
    value_scales = torch.empty_like(key_scales)
    storage = exact_sink_pages + exact_tail_pages
    exact_key = torch.zeros(batch * storage, PAGE, hkv, DIM, device=device, dtype=torch.float16)
    exact_value = torch.zeros_like(exact_key)
    old_counts, exact_idx, old_idx, exact_counts, last_len = [], [], [], [], []
    old_tokens, exact_tokens = [], []
    for r in range(batch):
        s, n = starts[r], pages[r]
        tok = lengths[r]
        flat_k = dense_k[s:s + n].reshape(-1, hkv, DIM)[:prefix_tokens[r]]
        flat_v = dense_v[s:s + n].reshape(-1, hkv, DIM)[:prefix_tokens[r]]
        key_center[r] = flat_k.float().mean(dim=0).half()
        value_center[r] = flat_v.float().mean(dim=0).half()
        d = dst[r]
        quantize_pages_into(dense_k[s:s + n], dense_v[s:s + n], key_center[r], value_center[r],
                            key_codes[d:d + n], value_codes[d:d + n], key_scales[d:d + n],
                            value_scales[d:d + n], 0, "half_away")
        n_old = max(n - exact_tail_pages - exact_sink_pages, 0)
        sink = min(exact_sink_pages, n)
        old_idx.extend(range(d + sink, d + sink + n_old))
        old_counts.append(n_old)
        ex_logical = list(range(sink)) + list(range(sink + n_old, n))
        ring = []
        for lp in ex_logical:
            slot = lp if lp < exact_sink_pages else exact_sink_pages + lp % exact_tail_pages
            phys = r * storage + slot
            exact_key[phys] = (dense_k[s + lp].float() - key_center[r][None].float()).half()
            exact_value[phys] = (dense_v[s + lp].float() - value_center[r][None].float()).half()
            ring.append(phys)
        exact_idx.extend(ring)
        exact_counts.append(len(ring))
        last_len.append((tok - 1) % PAGE + 1)
        old_tokens.append(n_old * PAGE)
        exact_tokens.append(tok - n_old * PAGE)

    def csr(counts):
        out = [0]
        for c in counts:
            out.append(out[-1] + c)
        return torch.tensor(out, dtype=torch.int32, device=device)

    tables = DecodeTables(
        old_indptr=csr(old_counts),
        old_indices=torch.tensor(old_idx or [0], dtype=torch.int32, device=device),
        exact_indptr=csr(exact_counts),
        exact_indices=torch.tensor(exact_idx or [0], dtype=torch.int32, device=device),
        exact_last_page_len=torch.tensor(last_len, dtype=torch.int32, device=device),
        old_tokens=old_tokens, exact_tokens=exact_tokens)
    cache = GaugeCache(exact_key, exact_value, key_codes, value_codes, key_scales, value_scales,
                       key_center, value_center, exact_tail_pages, exact_sink_pages)
    return cache, tables


def synthetic_dense_cache(lengths: list[int], hkv: int = 8, seed: int = 20261001,
                          device: torch.device | str = "cpu", theta: float = 1.0e6,
                          key_mean_var: float = 2.0, group: int = 4):
    """The benchmark's synthetic decode inputs: K = RoPE(N(mu_c, 1)) with
    mu_c ~ N(0, key_mean_var) per (head, channel), V ~ N(0, 1), Q ~ N(0, 1),
    request-major pages (the tail of a partial last page is zero-padded).
    Returns (q [B,group*hkv,128], dense_k, dense_v) as FP16 on ``device``."""
    gen = torch.Generator(device=device).manual_seed(seed)
    batch = len(lengths)
    pages = [math.ceil(n / PAGE) for n in lengths]
    total = sum(pages)
    mu = torch.randn(hkv, DIM, generator=gen, device=device) * math.sqrt(key_mean_var)
    q = torch.randn(batch, group * hkv, DIM, generator=gen, device=device).half()
    cos, sin = rope_tables(max(pages) * PAGE, theta, device=device)
    dense_k = torch.zeros(total, PAGE, hkv, DIM, device=device, dtype=torch.float16)
    dense_v = torch.zeros_like(dense_k)
    start = 0
    for r, n_tok in enumerate(lengths):
        k = (torch.randn(n_tok, hkv, DIM, generator=gen, device=device) + mu).half()
        v = torch.randn(n_tok, hkv, DIM, generator=gen, device=device).half()
        k = apply_rope_fp16(k, cos[:n_tok], sin[:n_tok])
        flat_k = dense_k[start:start + pages[r]].view(-1, hkv, DIM)
        flat_v = dense_v[start:start + pages[r]].view(-1, hkv, DIM)
        flat_k[:n_tok] = k
        flat_v[:n_tok] = v
        start += pages[r]
    return q, dense_k, dense_v
