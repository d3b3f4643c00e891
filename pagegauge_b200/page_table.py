"""Page-table helpers of the PageGauge decode path (host side).

Request-major physical storage; the exact FP16 storage of a request holds
``S`` fixed prefix pages, optional static-suffix pages, then a ring of
``T`` tail pages addressed by ``fixed + logical % T``.  Semantics and error
messages follow scripts/benchmark_page_gauge_transformer.py:383-667 and
segment_page_table in scripts/benchmark_flashinfer_page_affine_int8.py:392-420.
"""

from __future__ import annotations

from typing import Any

import torch

PAGE = 16


def request_major_page_table(batch_size: int, logical_page_capacity: int,
                             physical_pages_per_request: int | None = None,
                             device: torch.device | str = "cuda") -> torch.Tensor:
    """[B, P] map of logical page -> request-major physical page (:383-407)."""
    if batch_size <= 0 or logical_page_capacity <= 0:
        raise ValueError("batch size and page capacity must be positive")
    physical = logical_page_capacity if physical_pages_per_request is None else physical_pages_per_request
    if physical <= 0:
        raise ValueError("physical pages per request must be positive")
    logical = torch.arange(logical_page_capacity, device=device, dtype=torch.int32)
    offsets = torch.arange(batch_size, device=device, dtype=torch.int32) * physical
    return offsets[:, None] + logical.remainder(physical)[None, :]


def validate_exact_prefix_pages(exact_prefix_pages: int) -> int:
    if not isinstance(exact_prefix_pages, int) or exact_prefix_pages < 0:
        raise ValueError("exact prefix pages must be a nonnegative integer")
    return int(exact_prefix_pages)


def validate_exact_static_suffix_pages(exact_static_suffix_pages: int, *, exact_prefix_pages: int = 0,
                                       initial_context_pages: int | None = None) -> int:
    if not isinstance(exact_static_suffix_pages, int) or exact_static_suffix_pages < 0:
        raise ValueError("exact static suffix pages must be a nonnegative integer")
    if exact_static_suffix_pages:
        if initial_context_pages is None or initial_context_pages <= 0:
            raise ValueError("an exact static suffix requires positive initial context pages")
        if exact_prefix_pages + exact_static_suffix_pages >= initial_context_pages:
            raise ValueError("fixed exact prefix and suffix must leave an initial old-cache page")
    return int(exact_static_suffix_pages)


def validate_exact_prefix_attention_path(exact_prefix_pages: int, tail_attention: str) -> int:
    exact_prefix_pages = validate_exact_prefix_pages(exact_prefix_pages)
    if exact_prefix_pages and tail_attention != "flashinfer_merge":
        raise ValueError("exact prefix pages require the segmented flashinfer_merge path")
    return exact_prefix_pages


def _suffix_begin(static_suffix: int, initial_context_pages: int | None):
    return int(initial_context_pages) - static_suffix if static_suffix else None


def exact_physical_page_index(request: int, logical_page: int, exact_tail_pages: int,
                              exact_sink_pages: int = 0, exact_static_suffix_pages: int = 0,
                              initial_context_pages: int | None = None) -> int:
    """Logical page -> request-major fixed slot or tail-ring slot (:460-494)."""
    sink = validate_exact_prefix_pages(exact_sink_pages)
    suffix = validate_exact_static_suffix_pages(exact_static_suffix_pages, exact_prefix_pages=sink,
                                                initial_context_pages=initial_context_pages)
    if request < 0 or logical_page < 0 or exact_tail_pages <= 0:
        raise ValueError("exact page mapping inputs must be non-negative with a tail")
    fixed = sink + suffix
    begin = _suffix_begin(suffix, initial_context_pages)
    if logical_page < sink:
        local = logical_page
    elif begin is not None and begin <= logical_page < int(initial_context_pages):
        local = sink + logical_page - begin
    else:
        local = fixed + logical_page % exact_tail_pages
    return request * (fixed + exact_tail_pages) + local


def request_major_exact_page_table(batch_size: int, logical_page_capacity: int, exact_tail_pages: int,
                                   exact_sink_pages: int = 0, exact_static_suffix_pages: int = 0,
                                   initial_context_pages: int | None = None,
                                   device: torch.device | str = "cuda") -> torch.Tensor:
    """[B, P] map of every logical page to its exact slot (:497-533)."""
    sink = validate_exact_prefix_pages(exact_sink_pages)
    suffix = validate_exact_static_suffix_pages(exact_static_suffix_pages, exact_prefix_pages=sink,
                                                initial_context_pages=initial_context_pages)
    if batch_size <= 0 or logical_page_capacity <= 0 or exact_tail_pages <= 0:
        raise ValueError("batch, logical capacity, and exact tail must be positive")
    if sink >= logical_page_capacity:
        raise ValueError("exact prefix must be smaller than logical page capacity")
    logical = torch.arange(logical_page_capacity, device=device, dtype=torch.int32)
    fixed = sink + suffix
    local = fixed + logical.remainder(exact_tail_pages)
    if sink:
        local = torch.where(logical < sink, logical, local)
    if suffix:
        begin = initial_context_pages - suffix
        mask = (logical >= begin) & (logical < initial_context_pages)
        local = torch.where(mask, sink + logical - begin, local)
    offsets = torch.arange(batch_size, device=device, dtype=torch.int32) * (fixed + exact_tail_pages)
    return offsets[:, None] + local[None, :]


def page_gauge_logical_partition(total_pages: int, exact_tail_pages: int, exact_sink_pages: int,
                                 last_page_len: int, exact_static_suffix_pages: int = 0,
                                 initial_context_pages: int | None = None) -> dict[str, Any]:
    """Exact-once prefix / static suffix / old / tail partition (:536-599)."""
    sink = validate_exact_prefix_pages(exact_sink_pages)
    suffix = validate_exact_static_suffix_pages(exact_static_suffix_pages, exact_prefix_pages=sink,
                                                initial_context_pages=initial_context_pages)
    if total_pages <= 0 or exact_tail_pages <= 0:
        raise ValueError("total and exact-tail page counts must be positive")
    if not 1 <= last_page_len <= PAGE:
        raise ValueError("last page length lies outside one page")
    tail_begin = total_pages - exact_tail_pages
    if tail_begin <= sink:
        raise ValueError("context must contain at least one quantized old page")
    prefix = tuple(range(sink))
    suffix_pages = tuple(range(initial_context_pages - suffix, initial_context_pages)) if suffix else ()
    tail = tuple(range(tail_begin, total_pages))
    exact_set = set(prefix) | set(suffix_pages) | set(tail)
    old = tuple(p for p in range(total_pages) if p not in exact_set)
    exact = tuple(p for p in range(total_pages) if p in exact_set)
    union = old + exact
    disjoint = len(set(union)) == len(union) and set(union) == set(range(total_pages))
    context = (total_pages - 1) * PAGE + last_page_len
    old_tokens = len(old) * PAGE
    exact_tokens = context - old_tokens
    if not disjoint or old_tokens + exact_tokens != context:
        raise RuntimeError("PageGauge logical partition is not exact and disjoint")
    return {
        "prefix_logical_pages": prefix,
        "sink_logical_pages": prefix,
        "static_suffix_logical_pages": suffix_pages,
        "old_logical_pages": old,
        "tail_logical_pages": tail,
        "exact_logical_pages": exact,
        "tail_logical_begin": tail_begin,
        "old_page_count": len(old),
        "exact_page_count": len(exact),
        "old_token_count": old_tokens,
        "exact_token_count": exact_tokens,
        "context_token_count": context,
        "coverage_disjoint": disjoint,
    }


def write_exact_prefix_tail_page_table(destination: torch.Tensor, logical_to_exact_physical: torch.Tensor,
                                       tail_logical_begin: int, total_page_count: int,
                                       exact_sink_pages: int, exact_static_suffix_pages: int = 0,
                                       initial_context_pages: int | None = None) -> torch.Tensor:
    """Fixed prefix, static suffix, then the chronological tail (:602-667)."""
    sink = validate_exact_prefix_pages(exact_sink_pages)
    suffix = validate_exact_static_suffix_pages(exact_static_suffix_pages, exact_prefix_pages=sink,
                                                initial_context_pages=initial_context_pages)
    if destination.dtype != torch.int32 or logical_to_exact_physical.dtype != torch.int32:
        raise ValueError("exact page tables must use int32 indices")
    if destination.dim() != 2 or logical_to_exact_physical.dim() != 2:
        raise ValueError("exact page tables must have shape [B,P]")
    if int(destination.shape[0]) != int(logical_to_exact_physical.shape[0]):
        raise ValueError("exact page-table batch sizes differ")
    if not sink <= tail_logical_begin < total_page_count:
        raise ValueError("exact prefix and tail logical ranges overlap or are empty")
    if total_page_count > int(logical_to_exact_physical.shape[1]):
        raise ValueError("exact logical page table exceeds allocated capacity")
    begin = _suffix_begin(suffix, initial_context_pages)
    tail_pages = [p for p in range(tail_logical_begin, total_page_count)
                  if not (begin is not None and begin <= p < int(initial_context_pages))]
    active = sink + suffix + len(tail_pages)
    if active > int(destination.shape[1]):
        raise ValueError("exact active table exceeds destination capacity")
    if sink:
        destination[:, :sink].copy_(logical_to_exact_physical[:, :sink])
    cursor = sink
    if suffix:
        destination[:, cursor:cursor + suffix].copy_(logical_to_exact_physical[:, begin:initial_context_pages])
        cursor += suffix
    if tail_pages:
        idx = torch.tensor(tail_pages, device=logical_to_exact_physical.device, dtype=torch.long)
        destination[:, cursor:active].copy_(logical_to_exact_physical.index_select(1, idx))
    return destination[:, :active]


def write_exact_sink_tail_page_table(destination, logical_to_exact_physical, tail_logical_begin,
                                     total_page_count, exact_sink_pages):
    return write_exact_prefix_tail_page_table(destination, logical_to_exact_physical,
                                              tail_logical_begin, total_page_count, exact_sink_pages)


def write_page_gauge_old_page_table(destination: torch.Tensor, logical_to_physical: torch.Tensor,
                                    old_logical_pages: tuple[int, ...]) -> torch.Tensor:
    """Arbitrary exact-once old-page set in logical order (:670-696)."""
    if destination.dtype != torch.int32 or logical_to_physical.dtype != torch.int32:
        raise ValueError("old page tables must use int32 indices")
    if destination.dim() != 2 or logical_to_physical.dim() != 2:
        raise ValueError("old page tables must have shape [B,P]")
    if destination.shape[0] != logical_to_physical.shape[0]:
        raise ValueError("old page-table batch sizes differ")
    if not old_logical_pages:
        raise ValueError("old page set cannot be empty")
    if tuple(sorted(set(old_logical_pages))) != tuple(old_logical_pages):
        raise ValueError("old logical pages must be unique and increasing")
    if old_logical_pages[-1] >= int(logical_to_physical.shape[1]):
        raise ValueError("old logical page exceeds allocated capacity")
    if len(old_logical_pages) > int(destination.shape[1]):
        raise ValueError("old page set exceeds destination capacity")
    idx = torch.tensor(old_logical_pages, device=logical_to_physical.device, dtype=torch.long)
    destination[:, :len(old_logical_pages)].copy_(logical_to_physical.index_select(1, idx))
    return destination[:, :len(old_logical_pages)]


def write_heterogeneous_page_table(destination: torch.Tensor, old_pages: torch.Tensor,
                                   exact_ring_pages: torch.Tensor, old_page_count: int,
                                   total_page_count: int) -> torch.Tensor:
    """One logical table: code-page ids below ``old_page_count``, ring ids
    after it (:715-745)."""
    if destination.dtype != torch.int32:
        raise ValueError("heterogeneous page table must use int32 indices")
    if destination.dim() != 2 or old_pages.shape != destination.shape or exact_ring_pages.shape != destination.shape:
        raise ValueError("heterogeneous page tables must have matching [B,P] shapes")
    if not 0 <= old_page_count <= total_page_count <= int(destination.shape[1]):
        raise ValueError("heterogeneous page counts lie outside table capacity")
    if old_page_count:
        destination[:, :old_page_count].copy_(old_pages[:, :old_page_count])
    if old_page_count < total_page_count:
        destination[:, old_page_count:total_page_count].copy_(exact_ring_pages[:, old_page_count:total_page_count])
    return destination[:, :total_page_count]


def segment_page_table(pages_per_row: list[int], tail_pages: int, sink_pages: int = 0,
                       device: torch.device | str = "cuda"):
    """(old_indptr, old_indices, exact_indptr, exact_indices) for contiguous
    request-major storage (scripts/benchmark_flashinfer_page_affine_int8.py:392-420)."""
    old_counts = [max(c - tail_pages - sink_pages, 0) for c in pages_per_row]
    exact_counts = [c - o for c, o in zip(pages_per_row, old_counts)]
    old_idx: list[int] = []
    exact_idx: list[int] = []
    start = 0
    for count, old in zip(pages_per_row, old_counts):
        mid = start + sink_pages
        old_idx.extend(range(mid, mid + old))
        exact_idx.extend(range(start, mid))
        exact_idx.extend(range(mid + old, start + count))
        start += count

    def indptr(counts):
        acc, out = 0, [0]
        for c in counts:
            acc += c
            out.append(acc)
        return torch.tensor(out, device=device, dtype=torch.int32)

    return (indptr(old_counts), torch.tensor(old_idx, device=device, dtype=torch.int32),
            indptr(exact_counts), torch.tensor(exact_idx, device=device, dtype=torch.int32))
