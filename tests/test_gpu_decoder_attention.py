"""The decoder's PageGauge attention path at the benchmark decoder's layer
shape (configs[4]: hidden 4096, 32 query / 8 KV heads, FFN 14336, vocab
32768; two layers), isolated the way the reference compares its decoders
(the same model run with two attention implementations and the logit
sequences compared, scripts/benchmark_page_gauge_transformer.py:3306-3381).

Decoder A is the product: CUDA-graph steps with the split-KV PageGauge
kernels.  Decoder B is the same weights and the same cache after the same
prefill, stepped eagerly with the attention replaced by a plain PyTorch FP32
attention over that cache (INT8 pages dequantised as s*Z, the exact FP16
pages, softmax in FP32, plus the value centre).  Everything else -- the
projection GEMMs, norms, the fused append, the greedy head -- is the same
GPU code in both, so the logit difference is the attention path's.  B is
teacher-forced with A's tokens.  Bar, at every step (a 4096-token prompt,
20 steps crossing a page boundary): the logits computed in FP32 from each
decoder's final normalised hidden state (the LM head's input) within
max-abs 2e-3 and cosine >= 0.9999, and the FP16 logits the decoders emit
within 2e-3 plus one FP16 step of each other (at this width logits reach
8-16, where one FP16 step is 2^-7, so two independently rounded FP16 values
cannot be held to 2e-3 themselves).

Against the float64 decoder oracle this shape cannot be held to 2e-3: the
FP16 rounding of an independent forward at hidden 4096 alone puts logits
several 1e-3 apart (on the 2-layer, hidden-512 model the dense prefill,
which uses none of this library's kernels, is already 1.5e-3 from the
oracle).  tests/test_gpu_decoder.py compares with the oracle on that small
model."""

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
ATOL = 2e-3
MIN_COSINE = 0.9999
PAGE = 16


class TorchAttention:
    """Reference attention for decoder B: the decode call's arguments, the
    page tables of the decoder's current positions, FP32 torch maths."""

    def __init__(self, decoder: PageGaugeDecoder, real):
        self.decoder = decoder
        self.real = real

    def __getattr__(self, name):
        return getattr(self.real, name)

    def run(self, q, key_codes, value_codes, key_scales, value_scales, exact_key, exact_value,
            value_center, out=None, lse=None, **_):
        d = self.decoder
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

            k = tokens(key_codes, key_scales, exact_key)[:, kv_of_q]      # [T, Hq, 128]
            v = tokens(value_codes, value_scales, exact_value)[:, kv_of_q]
            s = torch.einsum("hd,thd->ht", q[r].float(), k) / math.sqrt(q.shape[2])
            o = torch.einsum("ht,thd->hd", torch.softmax(s, dim=1), v)
            o = o + value_center[r].float()[kv_of_q]
            out[r].copy_(o.half())
        return out


def _close(a: PageGaugeDecoder, b: PageGaugeDecoder, lm_head: torch.Tensor) -> float:
    got = a.normed.float() @ lm_head.float().t()
    exp = b.normed.float() @ lm_head.float().t()
    err = float((got - exp).abs().max())
    cos = float(torch.nn.functional.cosine_similarity(got.flatten(), exp.flatten(), dim=0))
    assert err <= ATOL and cos >= MIN_COSINE, f"max-abs {err:.3e} cosine {cos:.6f}"
    # FP16 logits: the same bar plus the two roundings to FP16 (half a step
    # each, the step at the larger value).
    la, lb = a.logits.float(), b.logits.float()
    big = torch.maximum(la.abs(), lb.abs()).clamp_min(2.0 ** -14)
    step = torch.exp2(torch.floor(torch.log2(big)) - 10)
    assert bool(((la - lb).abs() <= ATOL + step).all())
    return err


def test_decoder_attention_path_at_the_benchmark_layer_shape(cuda_lib):
    batch = 2
    weights = random_decoder_weights(CFG, 20261004, device="cuda")
    prompt = torch.randint(0, CFG.vocab, (batch, PROMPT),
                           generator=torch.Generator().manual_seed(41)).cuda()
    a = PageGaugeDecoder(weights, batch=batch, max_context=PROMPT + 64)
    b = PageGaugeDecoder(weights, batch=batch, max_context=PROMPT + 64)
    la = a.prefill(prompt)
    lb = b.prefill(prompt)
    torch.cuda.synchronize()
    assert torch.equal(la, lb)
    for ca, cb in zip(a.caches, b.caches):  # one cache state for both decoders
        for name in ("key_codes", "value_codes", "key_scales", "value_scales", "exact_key",
                     "exact_value", "key_center", "value_center"):
            getattr(cb, name).copy_(getattr(ca, name))
    entry = b._entry

    def torch_entry(positions):
        e = entry(positions)
        if not isinstance(e["dec"], TorchAttention):
            e["dec"] = TorchAttention(b, e["dec"])
        return e

    b._entry = torch_entry
    assert torch.equal(a.tokens, b.tokens)
    a.step(use_graph=True)  # A's first step runs eagerly (library warm-up), then graphs
    b.step(use_graph=False)
    worst = _close(a, b, weights.lm_head)
    crossed = False
    for _ in range(STEPS):
        b.tokens.copy_(a.tokens)  # teacher forcing: B embeds A's greedy token
        start_pages = int(a.host_positions[0]) // PAGE
        a.step(use_graph=True)
        b.step(use_graph=False)
        torch.cuda.synchronize()
        worst = max(worst, _close(a, b, weights.lm_head))
        crossed |= int(a.host_positions[0]) // PAGE != start_pages
    assert crossed and int(a.host_positions[0]) == PROMPT + STEPS + 1
    assert read_device_error() == 0
    print(f"worst logit max-abs {worst:.3e}")
