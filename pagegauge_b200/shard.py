"""Sharding a decode batch across the GPUs of one box (no data-path
collective).

Requests of a ragged decode batch are independent, and so are the KV heads
of a request, so a batch splits across ranks either way:

* by request: greedy longest-first bin packing on each request's decode
  bytes (INT8 old pages + scales + the FP16 exact tail); each rank decodes
  its own requests with its own cache;
* by KV head: every rank decodes every request over Hkv/N of its KV heads
  (and their query heads); each rank's bytes are exactly 1/N of the batch.

``plan_shards`` takes request shards when they balance the bytes to within
a tolerance and KV-head shards otherwise (a few long requests on many
GPUs).  Outputs are gathered on the host afterwards.  The reference runs
one GPU only; the per-request byte model is the one its B8 ragged
accounting uses (scripts/benchmark_flashinfer_page_affine_int8.py:392-420
splits old and exact pages per request).
"""

from __future__ import annotations

import heapq

import numpy as np

PAGE = 16
HEAD_DIM = 128


def ragged_lengths(batch: int, seed: int, low: int = 4096, high: int = 32768) -> list[int]:
    """Context lengths drawn uniform in [low, high] (the B8 ragged benchmark workload)."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(low, high + 1, size=batch)]


def request_bytes(length: int, exact_tail_tokens: int = 256, kv_heads: int = 8) -> int:
    """Algorithmic decode bytes of one request: INT8 K/V codes of the old
    full pages, their per-(page, head) FP16 K/V scales, and the FP16 K/V of
    the exact tokens (the last page may be partial; the tail covers it)."""
    exact_pages = min(-(-length // PAGE), -(-exact_tail_tokens // PAGE))
    old_pages = -(-length // PAGE) - exact_pages
    old_tokens = old_pages * PAGE
    exact_tokens = length - old_tokens
    return (2 * old_tokens * kv_heads * HEAD_DIM + old_pages * kv_heads * 2 * 2
            + 2 * exact_tokens * kv_heads * HEAD_DIM * 2)


def shard_requests(lengths, world: int, **kw) -> list[list[int]]:
    """Greedy longest-first assignment of request indices to ``world``
    ranks, minimising the largest per-rank byte total.  Deterministic:
    ties go to the lower rank; each rank's list is in request order."""
    if world < 1:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-request_bytes(lengths[i], **kw), i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + request_bytes(lengths[i], **kw), r))
    return [sorted(s) for s in shards]


def shard_loads(lengths, shards, **kw) -> list[int]:
    return [sum(request_bytes(lengths[i], **kw) for i in s) for s in shards]


def gather_outputs(shards, outputs, batch: int):
    """Place per-rank outputs (rows in each shard's request order) back
    into request order; ``outputs[r]`` is an array [len(shards[r]), ...]."""
    first = next(o for o in outputs if len(o))
    full = np.empty((batch,) + tuple(first.shape[1:]), dtype=first.dtype)
    for idx, out in zip(shards, outputs):
        for row, i in enumerate(idx):
            full[i] = out[row]
    return full


def head_range(kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """KV heads [h0, h1) of ``rank`` when ``world`` ranks split ``kv_heads``."""
    if world < 1 or kv_heads % world:
        raise ValueError("KV heads must divide evenly across the ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def plan_shards(lengths, world: int, kv_heads: int = 8, tolerance: float = 1.02) -> dict:
    """Choose how ``world`` ranks split a ragged batch: request shards when
    the largest rank's bytes are within ``tolerance`` of the mean (or the
    heads cannot be split evenly), else KV-head shards.  Returns
    {"mode": "requests" | "heads", "requests": [[request ids] per rank],
    "heads": [(h0, h1) per rank], "rank_bytes": [...]}."""
    shards = shard_requests(lengths, world, kv_heads=kv_heads)
    loads = shard_loads(lengths, shards, kv_heads=kv_heads)
    mean = sum(loads) / world
    if world == 1 or kv_heads % world or max(loads) <= mean * tolerance:
        return {"mode": "requests", "requests": shards,
                "heads": [(0, kv_heads)] * world, "rank_bytes": loads}
    per = kv_heads // world
    every = list(range(len(lengths)))
    return {"mode": "heads", "requests": [every] * world,
            "heads": [head_range(kv_heads, world, r) for r in range(world)],
            "rank_bytes": [sum(request_bytes(n, kv_heads=per) for n in lengths)] * world}


def gather_head_outputs(outputs, group: int):
    """Concatenate per-rank outputs [B, group * (Hkv/N), 128] of KV-head
    shards (rank order = head order) into [B, Hq, 128]."""
    return np.concatenate(list(outputs), axis=1)
