"""Mistral-shaped decoder whose attention is the PageGauge decode path
(the Mistral-7B-shaped benchmark decoder): random-init FP16 weights, a prompt prefill that
builds the page-gauge caches, then greedy decode steps captured in CUDA
graphs, optionally tensor-parallel over the GPUs of one box.

Per decode step and layer (the layer body of the reference's decoder,
scripts/benchmark_page_gauge_transformer.py:2754-2804, with its packed
projections, scripts/benchmark_e2e_transformer.py:149-233):

    residual += delta; x = RMSNorm(residual)            pg_add_rmsnorm
    qkv = x @ Wqkv^T                                      cuBLAS GEMM
    RoPE(q, k), centred append, page close               pg_rope_append_page_gauge_batched
    attn = PageGauge decode (INT8 old pages + FP16 ring)  pg_decode_run (split + merge, + c_V)
    o = attn @ Wo^T   [all-reduce over TP ranks]          cuBLAS GEMM (+ NCCL)
    residual += o; x = RMSNorm(residual)                 pg_add_rmsnorm
    act = SiLU(x @ Wg^T) * (x @ Wu^T)                    cuBLAS GEMM + pg_silu_mul
    delta = act @ Wd^T   [all-reduce over TP ranks]       cuBLAS GEMM (+ NCCL)

then RMSNorm, the LM head (vocabulary-parallel under TP) and a greedy
argmax; the next token's embedding starts the next step on the device.

Tensor parallelism shards by KV head (Megatron column-parallel qkv and
gate/up, row-parallel o and down, vocabulary-parallel LM head): rank t of T
holds KV heads [t*Hkv/T, (t+1)*Hkv/T) and their query heads, so every rank
runs the same PageGauge kernels on its own heads and caches.  The reference
is single-GPU; the sharding is this build's (tokens/s at 1/2/4/8 GPUs).

The caches follow build_caches (:1156-1259): per (layer, request, KV head)
centres are the FP32 mean of the prompt, every prompt page is quantised
with the completed-page quantiser, and the last 16 pages are kept centred
in FP16 in the request's ring (slot = page % 16).  Decode appends close
pages as they fill; a page leaves the exact window when its ring slot is
reused and is read from its INT8 copy from then on.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, scheduler
from .cache import GaugeCache, apply_rope_fp16, rope_tables
from .decode import PageGaugeDecode
from .gemm import RESIDUAL, SILU_MUL, STORE, PackedWeight, SkinnyGemm
from .peer import TpExchange
from .quantize import quantize_pages_into
from .runtime import load_append_extension

PAGE = 16
HEAD_DIM = 128


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    intermediate: int = 14336
    vocab: int = 32768
    rms_eps: float = 1e-5
    rope_theta: float = 1.0e6
    head_dim: int = HEAD_DIM

    @classmethod
    def mistral_7b_shaped(cls) -> "DecoderConfig":
        """The benchmark decoder: 32 layers, hidden 4096, 32/8 heads, FFN
        14336, vocab 32768, RoPE theta 1e6."""
        return cls()

    def parameter_count(self) -> int:
        attn = self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim \
            + self.heads * self.head_dim * self.hidden
        mlp = 3 * self.hidden * self.intermediate
        return self.layers * (attn + mlp + 2 * self.hidden) + 2 * self.vocab * self.hidden \
            + self.hidden


@dataclass(frozen=True)
class TensorParallel:
    """This rank's slices of the head, FFN and vocabulary dimensions."""

    rank: int
    world: int
    q_heads: tuple[int, int]
    kv_heads: tuple[int, int]
    intermediate: tuple[int, int]
    vocab: tuple[int, int]

    @classmethod
    def of(cls, cfg: DecoderConfig, rank: int = 0, world: int = 1) -> "TensorParallel":
        if world < 1 or not 0 <= rank < world:
            raise ValueError("bad tensor-parallel rank/world")
        if cfg.kv_heads % world or cfg.intermediate % (8 * world) or cfg.vocab % world:
            raise ValueError("KV heads, FFN width/8 and vocabulary must divide by the TP size")
        group = cfg.heads // cfg.kv_heads
        kv = cfg.kv_heads // world
        f = cfg.intermediate // world
        v = cfg.vocab // world
        return cls(rank, world, (rank * kv * group, (rank + 1) * kv * group),
                   (rank * kv, (rank + 1) * kv), (rank * f, (rank + 1) * f),
                   (rank * v, (rank + 1) * v))


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor  # [H]
    qkv: torch.Tensor        # [(hq_l + 2 hkv_l) * 128, H]  (q | k | v rows)
    o: torch.Tensor          # [H, hq_l * 128]
    mlp_norm: torch.Tensor   # [H]
    gate_up: torch.Tensor    # [2 F_l, H]  (gate | up rows)
    down: torch.Tensor       # [H, F_l]


@dataclass
class DecoderWeights:
    cfg: DecoderConfig
    tp: TensorParallel
    embed: torch.Tensor       # [V, H] (replicated)
    layers: list[LayerWeights] = field(default_factory=list)
    final_norm: torch.Tensor | None = None
    lm_head: torch.Tensor | None = None  # [V_l, H]


def full_layer_tensors(cfg: DecoderConfig, seed: int, layer: int, device, std: float = 0.02):
    """The unsharded FP16 tensors of one layer, N(0, std) weights and unit
    RMSNorm weights (transformers' Mistral initialisation), each from its own
    generator so every TP size slices the same model."""
    d = cfg.head_dim

    def randn(idx: int, *shape):
        g = torch.Generator(device=device).manual_seed(seed * 1000003 + layer * 101 + idx)
        return (torch.randn(*shape, generator=g, device=device) * std).half()

    return {
        "q": randn(0, cfg.heads * d, cfg.hidden),
        "k": randn(1, cfg.kv_heads * d, cfg.hidden),
        "v": randn(2, cfg.kv_heads * d, cfg.hidden),
        "o": randn(3, cfg.hidden, cfg.heads * d),
        "gate": randn(4, cfg.intermediate, cfg.hidden),
        "up": randn(5, cfg.intermediate, cfg.hidden),
        "down": randn(6, cfg.hidden, cfg.intermediate),
        "attn_norm": torch.ones(cfg.hidden, dtype=torch.float16, device=device),
        "mlp_norm": torch.ones(cfg.hidden, dtype=torch.float16, device=device),
    }


def full_model_tensors(cfg: DecoderConfig, seed: int, device, std: float = 0.02):
    g = torch.Generator(device=device).manual_seed(seed * 1000003 + 999_983)
    embed = (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=device) * std).half()
    g = torch.Generator(device=device).manual_seed(seed * 1000003 + 999_979)
    lm_head = (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=device) * std).half()
    return {"embed": embed, "lm_head": lm_head,
            "final_norm": torch.ones(cfg.hidden, dtype=torch.float16, device=device)}


def shard_layer(cfg: DecoderConfig, tp: TensorParallel, full: dict) -> LayerWeights:
    """Megatron slices of one layer for rank ``tp.rank``: column-parallel
    q/k/v and gate/up (rows of this rank's heads / FFN columns), row-parallel
    o and down (the matching input columns)."""
    d = cfg.head_dim
    q0, q1 = tp.q_heads
    k0, k1 = tp.kv_heads
    f0, f1 = tp.intermediate
    qkv = torch.cat((full["q"][q0 * d:q1 * d], full["k"][k0 * d:k1 * d],
                     full["v"][k0 * d:k1 * d]), 0).contiguous()
    gate_up = torch.cat((full["gate"][f0:f1], full["up"][f0:f1]), 0).contiguous()
    return LayerWeights(full["attn_norm"].contiguous(), qkv,
                        full["o"][:, q0 * d:q1 * d].contiguous(), full["mlp_norm"].contiguous(),
                        gate_up, full["down"][:, f0:f1].contiguous())


def random_decoder_weights(cfg: DecoderConfig, seed: int = 20261004, device="cuda",
                           tp: TensorParallel | None = None, gen_device=None,
                           std: float = 0.02) -> DecoderWeights:
    """This rank's shard of a random-init model (generated layer by layer on
    ``gen_device``, default ``device``, and moved to ``device``)."""
    tp = tp or TensorParallel.of(cfg)
    gen_device = gen_device or device
    top = full_model_tensors(cfg, seed, gen_device, std)
    v0, v1 = tp.vocab
    w = DecoderWeights(cfg, tp, top["embed"].to(device),
                       final_norm=top["final_norm"].to(device),
                       lm_head=top["lm_head"][v0:v1].contiguous().to(device))
    for layer in range(cfg.layers):
        full = full_layer_tensors(cfg, seed, layer, gen_device, std)
        lw = shard_layer(cfg, tp, full)
        w.layers.append(LayerWeights(*(t.to(device) for t in (
            lw.attn_norm, lw.qkv, lw.o, lw.mlp_norm, lw.gate_up, lw.down))))
        del full
    return w


def page_tables(positions, capacity_pages: int, ring_pages: int = 16, sink_pages: int = 0,
                suffix_pages: int = 0, initial_pages: int | None = None):
    """Per-request old/exact page lists for a decode step appending at
    ``positions[r]`` (the exact-once partition of
    page_gauge_logical_partition, scripts/benchmark_page_gauge_transformer.py:536-599):
    exact = the first ``sink_pages`` pages, the ``suffix_pages`` pages that
    ended the prompt (``initial_pages`` pages long), and the current page
    with the ``ring_pages - 1`` before it; every other page is INT8.  Exact
    pages map to exact_physical_page_index's slots (fixed slots, then the
    tail ring at ``fixed + page % ring_pages``), INT8 page p of request r to
    ``r * capacity_pages + p``.  Exact pages are listed in logical order, so
    the current (partial) page is last.  Returns CSR (old_indptr,
    old_indices, exact_indptr, exact_indices)."""
    from .page_table import exact_physical_page_index

    suffix_begin = (initial_pages - suffix_pages) if suffix_pages else None
    old_idx, ex_idx, old_cnt, ex_cnt = [], [], [0], [0]
    for r, p in enumerate(positions):
        total = int(p) // PAGE + 1
        tail_begin = max(0, total - ring_pages)
        n_old = n_ex = 0
        for lp in range(total):
            exact = (lp < sink_pages or lp >= tail_begin
                     or (suffix_begin is not None and suffix_begin <= lp < initial_pages))
            if exact:
                ex_idx.append(exact_physical_page_index(r, lp, ring_pages, sink_pages, suffix_pages,
                                                        initial_pages))
                n_ex += 1
            else:
                old_idx.append(r * capacity_pages + lp)
                n_old += 1
        old_cnt.append(old_cnt[-1] + n_old)
        ex_cnt.append(ex_cnt[-1] + n_ex)
    as32 = lambda x: np.asarray(x if len(x) else [0], dtype=np.int32)
    return (np.asarray(old_cnt, np.int32), as32(old_idx), np.asarray(ex_cnt, np.int32),
            as32(ex_idx))


def pick_greedy(pairs: torch.Tensor) -> torch.Tensor:
    """Global greedy token from per-rank (max logit, token id) pairs
    [world, B, 2] of vocabulary-parallel logits: the largest value, ties to
    the lowest rank (the lowest id, as argmax over the full row)."""
    best = torch.argmax(pairs[..., 0], dim=0)  # first maximum over ranks
    return pairs[..., 1].gather(0, best[None])[0].to(torch.int64)


def _call(name, *args):
    _lib.check(getattr(_lib.load(), name)(*args))


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class PageGaugeDecoder:
    """Greedy decoding with PageGauge attention on this rank's shard.

    ``process_group``: the tensor-parallel group (NCCL) or None for one GPU.
    ``tp_reduce`` (tensor parallelism, up to 32 rows): "peer" sums the
    row-parallel projections' partials through NVLink peer memory (the
    streaming GEMM publishes its tiles, or a small kernel publishes cuBLAS's
    output; the next kernel reduces and adds the residual + RMSNorm),
    "nccl" uses NCCL all-reduces.
    ``fuse_norm`` (one GPU, streaming GEMMs): compute the RMSNorms inside the
    qkv, gate/up and LM-head GEMMs instead of separate launches; measured
    slower on B200 (4.1-4.4 ms against 3.6-3.9 ms per B=1 step), so off by
    default.
    """

    def __init__(self, weights: DecoderWeights, batch: int, max_context: int,
                 process_group=None, ring_pages: int = 16, workspace_mb: int = 32,
                 gemm: str = "auto", sink_pages: int = 0, suffix_pages: int = 0,
                 fuse_norm: bool = False, tp_reduce: str = "peer"):
        cfg, tp = weights.cfg, weights.tp
        if cfg.head_dim != HEAD_DIM:
            raise ValueError("head_dim must be 128")
        self.cfg, self.tp, self.w = cfg, tp, weights
        self.pg = process_group
        self.fuse_norm = bool(fuse_norm)
        self.tpx = None
        self.batch = batch
        dev = weights.embed.device
        self.device = dev
        self.hq = tp.q_heads[1] - tp.q_heads[0]
        self.hkv = tp.kv_heads[1] - tp.kv_heads[0]
        self.inter = tp.intermediate[1] - tp.intermediate[0]
        self.vocab_local = tp.vocab[1] - tp.vocab[0]
        # Exact-page policy (the paper's S<sink>/A<suffix>/T<ring*16>): the
        # exact storage of a request is sink_pages fixed prefix slots,
        # suffix_pages slots for the pages that ended the prompt, then the
        # tail ring (page_table.exact_physical_page_index).
        from .page_table import validate_exact_prefix_pages
        self.ring_pages = ring_pages
        self.sink_pages = validate_exact_prefix_pages(sink_pages)
        self.suffix_pages = int(suffix_pages)
        if self.suffix_pages < 0 or ring_pages <= 0:
            raise ValueError("suffix pages must be non-negative and the ring positive")
        self.initial_pages = None
        self.fixed_pages = self.sink_pages + self.suffix_pages
        storage = self.fixed_pages + ring_pages
        self.capacity_pages = math.ceil(max_context / PAGE)
        self.max_context = self.capacity_pages * PAGE
        # FP32 accumulation in every cuBLAS reduction (no FP16 split-K sums).
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        B, cap, hkv = batch, self.capacity_pages, self.hkv
        z = dict(device=dev)
        self.caches: list[GaugeCache] = []
        for _ in range(cfg.layers):
            codes = lambda: torch.zeros(B * cap, PAGE, hkv, HEAD_DIM, dtype=torch.int8, **z)
            scales = lambda: torch.zeros(B * cap, hkv, dtype=torch.float16, **z)
            ring = lambda: torch.zeros(B * storage, PAGE, hkv, HEAD_DIM, dtype=torch.float16, **z)
            cen = lambda: torch.zeros(B, hkv, HEAD_DIM, dtype=torch.float16, **z)
            self.caches.append(GaugeCache(ring(), ring(), codes(), codes(), scales(), scales(),
                                          cen(), cen(), ring_pages, self.fixed_pages))
        self.cos, self.sin = rope_tables(self.max_context, cfg.rope_theta, device=dev)
        qkv_w = (self.hq + 2 * hkv) * HEAD_DIM
        h16 = dict(dtype=torch.float16, **z)
        self.residual = torch.zeros(B, cfg.hidden, **h16)
        self.normed = torch.zeros(B, cfg.hidden, **h16)
        self.qkv = torch.zeros(B, qkv_w, **h16)
        self.rq = torch.zeros(B, self.hq, HEAD_DIM, **h16)
        self.attn = torch.zeros(B, self.hq, HEAD_DIM, **h16)
        self.o = torch.zeros(B, cfg.hidden, **h16)
        self.gate_up = torch.zeros(B, 2 * self.inter, **h16)
        self.act = torch.zeros(B, self.inter, **h16)
        self.down = torch.zeros(B, cfg.hidden, **h16)
        self.logits = torch.zeros(B, self.vocab_local, **h16)
        self.best_val = torch.zeros(B, dtype=torch.float32, **z)
        self.best_idx = torch.zeros(B, dtype=torch.int64, **z)
        if gemm not in ("auto", "pg", "cublas"):
            raise ValueError("gemm must be 'auto', 'pg' (weight-streaming kernels) or 'cublas'")
        # Measured on B200: the weight-streaming kernels (fused epilogues,
        # PDL) win at up to 8 token rows; cuBLAS's tensor-core GEMMs win at 32.
        if gemm == "auto":
            gemm = "pg" if batch <= 8 else "cublas"
        self.gemm_impl = gemm
        self.sk = SkinnyGemm(dev)
        # Row-parallel o_proj / down_proj under tensor parallelism: "peer"
        # sums the ranks' partials through NVLink peer memory (the streaming
        # GEMM publishes its tiles; cuBLAS's output is published by a small
        # kernel) and adds the residual + RMSNorm in the same launch.
        if tp_reduce not in ("peer", "nccl"):
            raise ValueError("tp_reduce must be 'peer' or 'nccl'")
        if process_group is not None and tp_reduce == "peer" and batch <= 32:
            self.tpx = TpExchange(process_group, cfg.hidden // 64, dev)
        self.packed = []
        if gemm == "pg":
            # Weights in the streaming kernels' tiled layout (the row-major
            # copies stay for the dense prefill).
            for lw in weights.layers:
                self.packed.append({"qkv": PackedWeight(lw.qkv), "o": PackedWeight(lw.o),
                                    "gate_up": PackedWeight(lw.gate_up, SILU_MUL),
                                    "down": PackedWeight(lw.down)})
            self.lm_head_packed = PackedWeight(weights.lm_head)
            # o_proj / down_proj add into the residual in their epilogue; under
            # tensor parallelism they first sum the ranks' tiles through peer
            # memory (no NCCL all-reduce).
            tp = process_group is not None
            self.sk.reserve(qkv_w, cfg.hidden, B, STORE)
            self.sk.reserve(cfg.hidden, self.hq * HEAD_DIM, B, STORE if tp else RESIDUAL)
            self.sk.reserve(2 * self.inter, cfg.hidden, B, SILU_MUL)
            self.sk.reserve(cfg.hidden, self.inter, B, STORE if tp else RESIDUAL)
            self.sk.reserve(self.vocab_local, cfg.hidden, B, STORE)
        self.tokens = torch.zeros(B, dtype=torch.int64, **z)
        self.positions = torch.zeros(B, dtype=torch.int32, **z)
        self.last_len = torch.ones(B, dtype=torch.int32, **z)
        self.host_positions = np.zeros(B, dtype=np.int64)
        self.ext = load_append_extension()
        self._ws_bytes = workspace_mb << 20
        self._bank: dict = {}
        self._bank_size = 3
        self._warm = False
        self.stream = torch.cuda.Stream(device=dev)
        self._old_last = torch.full((B,), PAGE, dtype=torch.int32, **z)
        self.replans = 0

    # ----------------------------------------------------------- helpers
    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.pg is not None:
            torch.distributed.all_reduce(t, group=self.pg)

    def _norm(self, residual, delta, weight, out) -> None:
        _call("pg_add_rmsnorm", residual.data_ptr(), None if delta is None else delta.data_ptr(),
              weight.data_ptr(), out.data_ptr(), residual.shape[0], residual.shape[1],
              residual.stride(0), 0 if delta is None else delta.stride(0), out.stride(0),
              float(self.cfg.rms_eps), _stream())

    def _silu_mul(self, gate_up, out) -> None:
        _call("pg_silu_mul", gate_up.data_ptr(), out.data_ptr(), gate_up.shape[0], out.shape[1],
              gate_up.stride(0), out.stride(0), _stream())

    def _greedy(self, logits: torch.Tensor) -> torch.Tensor:
        """Argmax over the full vocabulary of vocabulary-parallel logits
        (ties to the lowest index, as torch.argmax on the full row)."""
        B = logits.shape[0]
        _call("pg_argmax_rows", logits.data_ptr(), logits.stride(0), B, logits.shape[1],
              self.tp.vocab[0], self.best_val.data_ptr(), self.best_idx.data_ptr(), _stream())
        vals, idx = self.best_val[:B], self.best_idx[:B]
        if self.pg is None:
            return idx
        pair = torch.stack((vals, idx.to(torch.float32)), dim=-1)  # [B, 2]; V < 2^24
        allp = torch.empty(self.tp.world, *pair.shape, dtype=pair.dtype, device=pair.device)
        torch.distributed.all_gather_into_tensor(allp, pair.contiguous(), group=self.pg)
        return pick_greedy(allp)

    # ----------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Dense prefill of ``prompt`` [B, T] (int64) request by request;
        builds every layer's page-gauge cache and returns the last-position
        logits of this rank's vocabulary slice [B, V_l] (FP16).  The first
        generated tokens are left in ``self.tokens``."""
        B, T = prompt.shape
        if B != self.batch or not 0 < T < self.max_context:
            raise ValueError("prompt must be [batch, T] with T below the cache capacity")
        pages = -(-T // PAGE)
        if self.suffix_pages:
            from .page_table import validate_exact_static_suffix_pages
            if T % PAGE:
                raise ValueError("a static exact suffix needs a page-aligned prompt")
            validate_exact_static_suffix_pages(self.suffix_pages, exact_prefix_pages=self.sink_pages,
                                               initial_context_pages=pages)
        self.initial_pages = pages
        out = torch.empty(B, self.vocab_local, dtype=torch.float16, device=self.device)
        for r in range(B):
            out[r] = self._prefill_request(r, prompt[r].to(self.device))
        self.logits.copy_(out)
        self.tokens.copy_(self._greedy(out))
        self.host_positions[:] = T
        self.positions.fill_(T)
        self.last_len.fill_(T % PAGE + 1)
        return out

    def _prefill_request(self, r: int, tokens: torch.Tensor) -> torch.Tensor:
        cfg, T = self.cfg, tokens.numel()
        d = HEAD_DIM
        h = self.w.embed.index_select(0, tokens).contiguous()
        x = torch.empty_like(h)
        delta = None
        cos, sin = self.cos[:T], self.sin[:T]
        group = self.hq // self.hkv
        for l, lw in enumerate(self.w.layers):
            self._norm(h, delta, lw.attn_norm, x)
            qkv = torch.matmul(x, lw.qkv.t())
            q = qkv[:, :self.hq * d].view(T, self.hq, d)
            k = qkv[:, self.hq * d:(self.hq + self.hkv) * d].view(T, self.hkv, d)
            v = qkv[:, (self.hq + self.hkv) * d:].view(T, self.hkv, d)
            q = apply_rope_fp16(q, cos, sin)
            k = apply_rope_fp16(k, cos, sin)
            self._fill_cache(l, r, k, v)
            kk = k.repeat_interleave(group, dim=1)
            vv = v.repeat_interleave(group, dim=1)
            att = torch.nn.functional.scaled_dot_product_attention(
                q.transpose(0, 1)[None], kk.transpose(0, 1)[None], vv.transpose(0, 1)[None],
                is_causal=True, scale=1.0 / math.sqrt(d))[0].transpose(0, 1).reshape(T, -1)
            o = torch.matmul(att, lw.o.t())
            self._all_reduce(o)
            self._norm(h, o, lw.mlp_norm, x)
            gu = torch.matmul(x, lw.gate_up.t())
            act = torch.empty(T, self.inter, dtype=torch.float16, device=self.device)
            self._silu_mul(gu, act)
            delta = torch.matmul(act, lw.down.t())
            self._all_reduce(delta)
        last = h[-1:].contiguous()
        self._norm(last, delta[-1:].contiguous(), self.w.final_norm, x[-1:])
        return torch.matmul(x[-1:], self.w.lm_head.t())[0]

    def _fill_cache(self, layer: int, r: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Centres, INT8 copies of every prompt page, and the FP16 ring of
        the last ring_pages pages (slot = page % ring_pages)."""
        c = self.caches[layer]
        T = k.shape[0]
        pages = -(-T // PAGE)
        dk = torch.zeros(pages * PAGE, self.hkv, HEAD_DIM, dtype=torch.float16, device=self.device)
        dv = torch.zeros_like(dk)
        dk[:T] = k
        dv[:T] = v
        c.key_center[r] = k.float().mean(0).half()
        c.value_center[r] = v.float().mean(0).half()
        base = r * self.capacity_pages
        dk = dk.view(pages, PAGE, self.hkv, HEAD_DIM)
        dv = dv.view(pages, PAGE, self.hkv, HEAD_DIM)
        quantize_pages_into(dk, dv, c.key_center[r], c.value_center[r],
                            c.key_codes[base:base + pages], c.value_codes[base:base + pages],
                            c.key_scales[base:base + pages], c.value_scales[base:base + pages],
                            0, "half_away")
        from .page_table import exact_physical_page_index
        suffix_begin = pages - self.suffix_pages
        for lp in range(pages):
            if not (lp < self.sink_pages or lp >= max(0, pages - self.ring_pages)
                    or (self.suffix_pages and lp >= suffix_begin)):
                continue
            slot = exact_physical_page_index(r, lp, self.ring_pages, self.sink_pages,
                                             self.suffix_pages, pages)
            c.exact_key[slot] = (dk[lp].float() - c.key_center[r].float()).half()
            c.exact_value[slot] = (dv[lp].float() - c.value_center[r].float()).half()

    # ------------------------------------------------------------ decode
    def _entry(self, positions) -> dict:
        """The plan (work list + page tables + captured step) of the page
        structure of ``positions``: plans are kept per structure, like the
        reference's structural graph banks
        (scripts/benchmark_page_gauge_transformer.py:3026-3157), so a step
        whose structure was prepared replays without planning or capture."""
        key = tuple(int(p) // PAGE for p in positions)
        entry = self._bank.get(key)
        if entry is not None:
            self._bank[key] = self._bank.pop(key)  # most recently used last
            return entry
        if max(int(p) for p in positions) >= self.max_context:
            raise RuntimeError("decode position exceeds the cache capacity")
        o_ptr, o_idx, e_ptr, e_idx = page_tables(positions, self.capacity_pages, self.ring_pages,
                                                 self.sink_pages, self.suffix_pages,
                                                 self.initial_pages)
        dev = self.device
        dec = PageGaugeDecode(torch.empty(self._ws_bytes, dtype=torch.uint8, device=dev))
        old_idx = torch.from_numpy(o_idx).to(dev)
        ex_idx = torch.from_numpy(e_idx).to(dev)
        has_old = bool(o_ptr[-1] > 0)
        split = scheduler.lookup(self.batch, int(max(positions)) + 1, kv_heads=self.hkv)
        dec.plan(torch.from_numpy(o_ptr) if has_old else None, old_idx if has_old else None,
                 torch.from_numpy(e_ptr), ex_idx, self.last_len, self.hq, self.hkv,
                 old_split_pages=split, old_last_page_len=self._old_last if has_old else None)
        entry = {"dec": dec, "old": old_idx, "exact": ex_idx, "graph": None}
        self._bank[key] = entry
        while len(self._bank) > self._bank_size:
            self._bank.pop(next(iter(self._bank)))
        self.replans += 1
        return entry

    def _step_body(self, dec: PageGaugeDecode) -> None:
        """One decode step on the current stream (capturable)."""
        d = HEAD_DIM
        B = self.batch
        torch.index_select(self.w.embed, 0, self.tokens, out=self.residual)
        q_w, kv_w = self.hq * d, self.hkv * d
        fused = self.gemm_impl == "pg" and (self.pg is None or self.tpx is not None)
        fuse_norm = fused and self.fuse_norm and self.pg is None
        tpx = self.tpx
        pending = False  # a published down_proj awaits its peer reduction
        delta = None
        eps = self.cfg.rms_eps
        for l, lw in enumerate(self.w.layers):
            c = self.caches[l]
            pk = self.packed[l] if self.packed else {}
            if fuse_norm:
                # RMSNorm inside the qkv projection.
                self.sk(self.residual, pk["qkv"], out=self.qkv, norm_weight=lw.attn_norm, eps=eps)
            else:
                if pending:
                    # residual += sum of the ranks' down_proj tiles, then RMSNorm.
                    tpx.reduce(B, self.residual, lw.attn_norm, eps, self.normed)
                else:
                    self._norm(self.residual, delta, lw.attn_norm, self.normed)
                self._linear(self.normed, lw.qkv, self.qkv, pk.get("qkv"))
            q = self.qkv[:, :q_w].view(B, self.hq, d)
            k = self.qkv[:, q_w:q_w + kv_w].view(B, self.hkv, d)
            v = self.qkv[:, q_w + kv_w:].view(B, self.hkv, d)
            self.ext.rope_append_page_gauge_batched(
                q, k, v, self.cos, self.sin, self.positions, c.key_center, c.value_center,
                self.rq, c.exact_key, c.exact_value, c.key_codes, c.value_codes, c.key_scales,
                c.value_scales, self.fixed_pages)
            # With a one-page ring the page this step's append closes is
            # INT8 at the next step, whose decode must then wait for it.
            dec.run(self.rq, c.key_codes, c.value_codes, c.key_scales, c.value_scales,
                    c.exact_key, c.exact_value, c.value_center, out=self.attn,
                    int8_after_wait=self.ring_pages == 1)
            if fused and tpx is not None:
                # Row-parallel projections publish their tiles through peer
                # memory; the next kernel sums the ranks' tiles into the
                # residual and normalises (no NCCL all-reduce).
                self.sk(self.attn.view(B, -1), pk["o"], tp=tpx)
                tpx.reduce(B, self.residual, lw.mlp_norm, eps, self.normed)
                self.sk(self.normed, pk["gate_up"], out=self.act, mode=SILU_MUL)
                self.sk(self.act, pk["down"], tp=tpx)
                pending = True
                continue
            if fused:
                # residual += attn @ Wo^T (fused epilogue), then the MLP with
                # SiLU(gate) * up fused into the gate/up projection and the
                # down projection added into the residual.
                self.sk(self.attn.view(B, -1), pk["o"], mode=RESIDUAL, residual=self.residual)
                if fuse_norm:
                    self.sk(self.residual, pk["gate_up"], out=self.act, mode=SILU_MUL,
                            norm_weight=lw.mlp_norm, eps=eps)
                else:
                    self._norm(self.residual, None, lw.mlp_norm, self.normed)
                    self.sk(self.normed, pk["gate_up"], out=self.act, mode=SILU_MUL)
                self.sk(self.act, pk["down"], mode=RESIDUAL, residual=self.residual)
                delta = None
                continue
            self._linear(self.attn.view(B, -1), lw.o, self.o, pk.get("o"))
            if tpx is not None:
                # cuBLAS partials through peer memory: publish, then sum +
                # residual + RMSNorm in one launch.
                tpx.publish(self.o)
                tpx.reduce(B, self.residual, lw.mlp_norm, eps, self.normed)
            else:
                self._all_reduce(self.o)
                self._norm(self.residual, self.o, lw.mlp_norm, self.normed)
            if self.gemm_impl == "pg":
                self.sk(self.normed, pk["gate_up"], out=self.act, mode=SILU_MUL)
            else:
                torch.matmul(self.normed, lw.gate_up.t(), out=self.gate_up)
                self._silu_mul(self.gate_up, self.act)
            self._linear(self.act, lw.down, self.down, pk.get("down"))
            if tpx is not None:
                tpx.publish(self.down)
                pending = True
                continue
            self._all_reduce(self.down)
            delta = self.down
        if fuse_norm:
            self.sk(self.residual, self.lm_head_packed, out=self.logits,
                    norm_weight=self.w.final_norm, eps=eps)
        else:
            if pending:
                tpx.reduce(B, self.residual, self.w.final_norm, eps, self.normed)
            else:
                self._norm(self.residual, delta, self.w.final_norm, self.normed)
            self._linear(self.normed, self.w.lm_head, self.logits,
                         self.lm_head_packed if self.packed else None)
        self.tokens.copy_(self._greedy(self.logits))
        _call("pg_step_positions", self.positions.data_ptr(), self.last_len.data_ptr(), B, 1,
              _stream())

    def _linear(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
                packed: PackedWeight | None = None) -> None:
        if packed is not None:
            self.sk(x, packed, out=out)
        else:
            torch.matmul(x, w.t(), out=out)

    def launches_per_step(self) -> int:
        """Kernel launches of this library in one decode step."""
        entry = next(iter(self._bank.values()), None)
        attn = 2
        if entry is not None:
            plan = entry["dec"].work_plan
            attn = 1 if (plan.single and plan.num_items) else 2
        if self.gemm_impl == "pg" and self.pg is None and self.fuse_norm:
            # qkv (+RMSNorm), append, o (+residual), gate_up (+RMSNorm,
            # SiLU), down (+residual) per layer; the LM head (+final norm),
            # argmax and position update.
            return self.cfg.layers * (5 + attn) + 3
        if self.gemm_impl == "pg":
            # norm, qkv, append, o (+residual; under TP with the ranks'
            # reduction), norm, gate_up (+SiLU), down (+residual, same) per
            # layer; the final norm, LM head, argmax and position update.
            return self.cfg.layers * (7 + attn) + 4
        if self.tpx is not None:
            # cuBLAS projections with the peer-memory reduction: norm (or
            # reduce), append, attention, publish o, reduce (+residual,
            # RMSNorm), SiLU*up, publish down per layer.
            return self.cfg.layers * (6 + attn) + 3
        return self.cfg.layers * (4 + attn) + 3

    def _capture(self, entry: dict) -> None:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self._step_body(entry["dec"])
        entry["graph"] = graph

    def close(self) -> None:
        """Collective under tensor parallelism: release the peer-memory
        exchange buffers (before the process group is destroyed)."""
        self._bank.clear()
        if self.tpx is not None:
            self.tpx.close()
            self.tpx = None

    @torch.no_grad()
    def prepare(self, steps: int) -> int:
        """Plan and capture the steps' page structures ahead of time (after
        one eager step has initialised cuBLAS/NCCL on the decode stream).
        Returns how many new graphs were captured."""
        if not self._warm:
            raise RuntimeError("run one eager step before preparing graphs")
        n = 0
        with torch.cuda.stream(self.stream):
            for i in range(steps):
                entry = self._entry(self.host_positions + i)
                if entry["graph"] is None:
                    self._capture(entry)
                    n += 1
        return n

    @torch.no_grad()
    def step(self, use_graph: bool = True) -> torch.Tensor:
        """Append the current tokens at the current positions, attend, and
        leave the next greedy tokens in ``self.tokens`` (on ``self.stream``;
        the caller's stream is ordered around it)."""
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            entry = self._entry(self.host_positions)
            if use_graph and self._warm:
                if entry["graph"] is None:
                    self._capture(entry)
                entry["graph"].replay()
            else:
                self._step_body(entry["dec"])
                self._warm = True
        torch.cuda.current_stream().wait_stream(self.stream)
        self.host_positions += 1
        return self.tokens

    @torch.no_grad()
    def generate(self, steps: int, use_graph: bool = True) -> torch.Tensor:
        """``steps`` greedy decode steps; returns the generated tokens
        [steps, B] on the device (the prefill's token is not included)."""
        out = torch.empty(steps, self.batch, dtype=torch.int64, device=self.device)
        for i in range(steps):
            self.step(use_graph)
            out[i].copy_(self.tokens)
        return out
