"""Request sharding across the GPUs of one box (no data-path collective).

Requests of a ragged decode batch are independent, so a batch is split
across ranks by greedy longest-first bin packing on each request's decode
bytes (INT8 old pages + scales + the FP16 exact tail); each rank decodes
its own requests with its own cache and the outputs are gathered on the
host afterwards.  The reference runs one GPU only; the per-request byte
model is the one its B8 ragged accounting uses
(scripts/benchmark_flashinfer_page_affine_int8.py:392-420 splits old and
exact pages per request).
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
