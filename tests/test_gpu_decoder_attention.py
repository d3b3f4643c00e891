"""The decoder's PageGauge attention at the benchmark decoder's layer shape
(configs[4]: hidden 4096, 32 query / 8 KV heads, FFN 14336, vocab 32768;
two layers, a 4096-token prompt, 20 greedy steps crossing a page boundary).

Three decoders share the weights and the cache the prefill built:

* A runs its steps eagerly and, at every layer of every step, runs the
  PageGauge decode (split-KV kernel + merge + value centre) and a plain
  PyTorch FP32 attention over the same query and cache (INT8 pages
  dequantised as s*Z, the exact FP16 pages, softmax in FP32, plus the value
  centre); the two outputs must agree within max-abs 2e-3 and cosine
  >= 0.9999, the parity bar for attention outputs.
* A' is the product as the benchmark runs it (CUDA-graph steps); its logits
  must equal A's bit for bit, so what was checked is what runs.
* B replaces the PageGauge decode with the FP32 torch attention (the
  reference's method: one model, two attention implementations, logit
  sequences compared, scripts/benchmark_page_gauge_transformer.py:3306-3381),
  teacher-forced with A's tokens.  The logits computed in FP32 from each
  decoder's final normalised hidden state must have cosine >= 0.9999 and
  max-abs <= 1e-2.  The absolute logit bar cannot be 2e-3 at this width:
  once any attention output differs in its last FP16 bit, the FP16 residual
  stream flips last bits in a random subset of its 4096 elements, which
  moves N(0, 0.02)-weight logits by about 6e-4 each (sqrt(4096) * 5e-4 *
  0.02), about 3e-3 at the maximum over 65,536 logits, and two layers of
  FFN double that.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from pagegauge_b200.decoder import (DecoderConfig, PageGaugeDecoder, page_tables,
                                    random_decoder_weights)
from pagegauge_b200.runtime import read_device_error

pytestmark = pytest.mark.gpu

CFG = DecoderConfig(layers=2, hidden=4096, heads=32, kv_heads=8, intermediate=14336,
                    vocab=32768)
PROMPT = 4096
STEPS = 20
PAGE = 16
ATTN_ATOL = 2e-3
MIN_COSINE = 0.9999
LOGIT_ATOL = 1e-2


def torch_attention(d: PageGaugeDecoder, q, key_codes, value_codes, key_scales, value_scales,
                    exact_key, exact_value, value_center, out) -> None:
    """FP32 attention over the decoder's cache at its current positions."""
    positions = [int(p) for p in d.host_positions]
    o_ptr, o_idx, e_ptr, e_idx = page_tables(positions, d.capacity_pages, d.ring_pages,
                                             d.sink_pages, d.suffix_pages, d.initial_pages)
    group = q.shape[1] // key_codes.shape[2]
    kv_of_q = torch.arange(q.shape[1], device=q.device) // group
    for r, p in enumerate(positions):
        old = torch.from_numpy(o_idx[o_ptr[r]:o_ptr[r + 1]].astype(np.int64)).to(q.device)
        ex = torch.from_numpy(e_idx[e_ptr[r]:e_ptr[r + 1]].astype(np.int64)).to(q.device)
        n_ex = p + 1 - PAGE * len(old)

        def tokens(codes, scales, exact):
            deq = codes[old].float() * scales[old].float()[:, None, :, None]
            return torch.cat([deq.reshape(-1, *codes.shape[2:]),
                              exact[ex].float().reshape(-1, *codes.shape[2:])[:n_ex]])

        k = tokens(key_codes, key_scales, exact_key)[:, kv_of_q]  # [T, Hq, 128]
        v = tokens(value_codes, value_scales, exact_value)[:, kv_of_q]
        s = torch.einsum("hd,thd->ht", q[r].float(), k) / math.sqrt(q.shape[2])
        o = torch.einsum("ht,thd->hd", torch.softmax(s, dim=1), v)
        out[r].copy_((o + value_center[r].float()[kv_of_q]).half())


class Attention:
    """Stands in for a decoder's PageGaugeDecode object: ``mode`` "checked"
    runs the product and compares it with torch on the same call; "torch"
    runs torch only."""

    def __init__(self, decoder: PageGaugeDecoder, real, mode: str, record: list):
        self.decoder, self.real, self.mode, self.record = decoder, real, mode, record

    def __getattr__(self, name):
        return getattr(self.real, name)

    def run(self, q, key_codes, value_codes, key_scales, value_scales, exact_key, exact_value,
            value_center, out=None, lse=None, **kw):
        args = (q, key_codes, value_codes, key_scales, value_scales, exact_key, exact_value,
                value_center)
        if self.mode == "torch":
            torch_attention(self.decoder, *args, out)
            return out
        self.real.run(*args, out=out, lse=lse, **kw)
        ref = torch.empty_like(out)
        torch_attention(self.decoder, *args, ref)
        got, exp = out.float(), ref.float()
        self.record.append((float((got - exp).abs().max()),
                            float(torch.nn.functional.cosine_similarity(got.flatten(),
                                                                        exp.flatten(), dim=0))))
        return out


def _swap_attention(dec: PageGaugeDecoder, mode: str, record: list) -> None:
    entry = dec._entry

    def wrapped(positions):
        e = entry(positions)
        if not isinstance(e["dec"], Attention):
            e["dec"] = Attention(dec, e["dec"], mode, record)
        return e

    dec._entry = wrapped


def test_decoder_attention_path_at_the_benchmark_layer_shape(cuda_lib):
    batch = 2
    weights = random_decoder_weights(CFG, 20261004, device="cuda")
    prompt = torch.randint(0, CFG.vocab, (batch, PROMPT),
                           generator=torch.Generator().manual_seed(41)).cuda()
    decs = [PageGaugeDecoder(weights, batch=batch, max_context=PROMPT + 64) for _ in range(3)]
    first = [d.prefill(prompt) for d in decs]
    torch.cuda.synchronize()
    assert all(torch.equal(first[0], f) for f in first[1:])
    a, a_graph, b = decs
    for other in (a_graph, b):  # one cache state for all three
        for ca, cb in zip(a.caches, other.caches):
            for name in ("key_codes", "value_codes", "key_scales", "value_scales",
                         "exact_key", "exact_value", "key_center", "value_center"):
                getattr(cb, name).copy_(getattr(ca, name))
    checks: list = []
    _swap_attention(a, "checked", checks)
    _swap_attention(b, "torch", [])
    lm = weights.lm_head.float()
    worst_logit = 0.0
    crossed = False
    for i in range(STEPS + 1):
        b.tokens.copy_(a.tokens)  # teacher forcing
        start_page = int(a.host_positions[0]) // PAGE
        a.step(use_graph=False)
        a_graph.step(use_graph=True)
        b.step(use_graph=False)
        torch.cuda.synchronize()
        assert torch.equal(a.logits, a_graph.logits), f"graph step {i} differs from eager"
        got, exp = a.normed.float() @ lm.t(), b.normed.float() @ lm.t()
        err = float((got - exp).abs().max())
        cos = float(torch.nn.functional.cosine_similarity(got.flatten(), exp.flatten(), dim=0))
        assert err <= LOGIT_ATOL and cos >= MIN_COSINE, f"step {i}: logits {err:.3e} {cos:.6f}"
        worst_logit = max(worst_logit, err)
        crossed |= int(a.host_positions[0]) // PAGE != start_page
    assert len(checks) == (STEPS + 1) * CFG.layers
    worst = max(c[0] for c in checks)
    lowest_cos = min(c[1] for c in checks)
    assert worst <= ATTN_ATOL and lowest_cos >= MIN_COSINE, (worst, lowest_cos)
    assert crossed and int(a.host_positions[0]) == PROMPT + STEPS + 1
    assert read_device_error() == 0
    print(f"attention max-abs {worst:.3e} (cosine >= {lowest_cos:.7f}); "
          f"logits max-abs {worst_logit:.3e}")
