"""Single-launch-family ABI of the heterogeneous PageGauge decode
(scripts/page_gauge_heterogeneous_fa2.py:249-379): one logical page table
whose entries below ``old_kv_len`` are INT8 code pages and later entries are
centred FP16 ring pages; the value centre is restored in the epilogue.

On B200 the two page kinds are planned as separate work items of one split-
KV launch, so no tile mixes INT8 and FP16 and no shared-memory repacking is
needed; a merge launch combines the splits and adds c_V.
"""

from __future__ import annotations

import math
from typing import Any

import numpy as np
import torch

from .wrapper import (HEAD_DIM, PAGE, PagedDecodePlan, _segment, _Workspace, host_indptr,
                      launch_decode, num_sms, plan_items)

HQ = 32
HKV = 8
DIM = HEAD_DIM


class HeterogeneousDecodeWrapper:
    def __init__(self, workspace: torch.Tensor, use_cuda_graph: bool = False,
                 paged_kv_indptr_buffer=None, paged_kv_indices_buffer=None,
                 paged_kv_last_page_len_buffer=None, **_ignored):
        self._ws = _Workspace(workspace)
        self._use_cuda_graph = use_cuda_graph
        self._buffers = (paged_kv_indptr_buffer, paged_kv_indices_buffer, paged_kv_last_page_len_buffer)
        self._indptr_host: np.ndarray | None = None
        self._old_key: tuple | None = None
        self._plan: PagedDecodePlan | None = None
        self._split = 0
        self.page_gauge_module_uri = "pagegauge_b200.sm100a.heterogeneous"

    def plan(self, indptr, indices, last_page_len, num_qo_heads=HQ, num_kv_heads=HKV,
             head_dim=DIM, page_size=PAGE, fixed_split_size=None, old_kv_len=None, **_ignored):
        if (num_qo_heads, num_kv_heads, head_dim, page_size) != (HQ, HKV, DIM, PAGE):
            raise ValueError("heterogeneous decode supports Hq/Hkv=32/8, D128, page16")
        self._indptr_host = host_indptr(indptr)
        batch = self._indptr_host.size - 1
        if self._use_cuda_graph:
            ib, xb, lb = self._buffers
            nnz = int(self._indptr_host[-1])
            ib[: batch + 1].copy_(indptr)
            if xb.data_ptr() != indices.data_ptr():
                xb[:nnz].copy_(indices[:nnz])
            if lb.data_ptr() != last_page_len.data_ptr():
                lb[:batch].copy_(last_page_len)
            indices, last_page_len = xb, lb
        self._indices = indices
        self._last = last_page_len
        self._split = int(fixed_split_size or 0)
        self._full = torch.full((batch,), PAGE, dtype=torch.int32, device=indices.device)
        self._old_key = None
        if old_kv_len is not None:
            self._prepare(np.asarray(old_kv_len, dtype=np.int64).reshape(-1))

    def _prepare(self, old_tokens: np.ndarray) -> None:
        key = tuple(int(x) for x in old_tokens)
        if key == self._old_key:
            return
        ind = self._indptr_host
        batch = ind.size - 1
        old_pages = old_tokens // PAGE
        counts = np.diff(ind)
        if np.any(old_pages > counts):
            raise ValueError("old_kv_len exceeds the planned page count")
        # Compact the unified table into one CSR per page kind (device gather).
        starts = ind[:-1]
        old_sel = np.concatenate([np.arange(s, s + o) for s, o in zip(starts, old_pages)]) if batch else []
        ex_sel = np.concatenate([np.arange(s + o, s + c) for s, o, c in zip(starts, old_pages, counts)])
        dev = self._indices.device
        self._old_idx = self._indices[torch.as_tensor(np.asarray(old_sel, np.int64), device=dev)].contiguous() \
            if len(old_sel) else torch.zeros(1, dtype=torch.int32, device=dev)
        self._ex_idx = self._indices[torch.as_tensor(np.asarray(ex_sel, np.int64), device=dev)].contiguous() \
            if len(ex_sel) else torch.zeros(1, dtype=torch.int32, device=dev)
        o_ind = np.concatenate([[0], np.cumsum(old_pages)]).astype(np.int32)
        e_ind = np.concatenate([[0], np.cumsum(counts - old_pages)]).astype(np.int32)
        items, off, info = plan_items(batch, HKV, o_ind, e_ind, self._split, self._split,
                                      num_sms(dev))
        self._plan = PagedDecodePlan(self._ws, items, off, info, batch, HKV, HQ // HKV)
        self._old_key = key

    def run(self, q, paged_kv_cache, k_page_scale, v_page_scale, exact_k_cache, exact_v_cache,
            old_kv_len, value_center, sm_scale=None, out=None, lse=None, return_lse=False,
            int8_after_wait=False, **_ignored):
        """``int8_after_wait``: see PageGaugeDecode.run (a page closed by the
        append just before this call is read here as INT8)."""
        if self._indptr_host is None:
            raise RuntimeError("plan() must be called before run()")
        if self._old_key is None:
            self._prepare(old_kv_len.detach().to("cpu", torch.int64).numpy())
        old_k, old_v = paged_kv_cache
        if out is None:
            out = torch.empty_like(q)
        if lse is None and return_lse:
            lse = torch.empty(q.shape[0], HQ, device=q.device, dtype=torch.float32)
        segs = (_segment(old_k, old_v, self._old_idx, self._full, k_page_scale, v_page_scale),
                _segment(exact_k_cache, exact_v_cache, self._ex_idx, self._last))
        launch_decode(self._plan, q, segs, 1.0 / math.sqrt(DIM) if sm_scale is None else sm_scale,
                      out, lse, value_center=value_center, int8_after_wait=int8_after_wait)
        return (out, lse) if return_lse else out


def make_heterogeneous_page_gauge_wrapper(flashinfer: Any, workspace: torch.Tensor, **wrapper_kwargs):
    if workspace.device.type != "cuda" or workspace.dtype != torch.uint8:
        raise ValueError("workspace must be a CUDA uint8 tensor")
    wrapper_kwargs.pop("jit_args", None)
    return HeterogeneousDecodeWrapper(workspace, **wrapper_kwargs)


def plan_decode(wrapper, indptr, indices, last_page_len, *, fixed_split_pages: int = 0,
                old_kv_len=None) -> None:
    """scripts/page_gauge_heterogeneous_fa2.py:249-283."""
    for name, tensor in (("indptr", indptr), ("indices", indices), ("last_page_len", last_page_len)):
        if tensor.device.type != "cuda" or tensor.dtype != torch.int32 or not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous CUDA int32")
    if indptr.ndim != 1 or last_page_len.shape != (indptr.numel() - 1,):
        raise ValueError("indptr/last_page_len batch dimensions disagree")
    if fixed_split_pages < 0:
        raise ValueError("fixed_split_pages must be non-negative")
    wrapper.plan(indptr, indices, last_page_len, HQ, HKV, DIM, PAGE,
                 fixed_split_size=fixed_split_pages or None, old_kv_len=old_kv_len)


def validate_run_inputs(query, old_k_cache, old_v_cache, k_page_scale, v_page_scale,
                        exact_k_cache, exact_v_cache, old_kv_len, value_center) -> None:
    """scripts/page_gauge_heterogeneous_fa2.py:286-328 (same messages)."""
    batch = int(query.shape[0]) if query.ndim == 3 else -1
    if tuple(query.shape) != (batch, HQ, DIM) or query.dtype != torch.float16:
        raise ValueError(f"query must have decode-only shape [B,{HQ},{DIM}] and dtype float16")
    if query.device.type != "cuda" or not query.is_contiguous():
        raise ValueError("query must be contiguous CUDA storage")
    for name, cache, dtype in (("old_k_cache", old_k_cache, torch.int8), ("old_v_cache", old_v_cache, torch.int8),
                               ("exact_k_cache", exact_k_cache, torch.float16),
                               ("exact_v_cache", exact_v_cache, torch.float16)):
        if (cache.device.type != "cuda" or cache.dtype != dtype or cache.ndim != 4
                or tuple(cache.shape[1:]) != (PAGE, HKV, DIM) or not cache.is_contiguous()):
            raise ValueError(f"{name} must be contiguous CUDA [{name.split('_')[0]}_pages,16,8,128] {dtype}")
    if old_k_cache.shape != old_v_cache.shape or exact_k_cache.shape != exact_v_cache.shape:
        raise ValueError("K/V cache shapes must match within each representation")
    for name, scale in (("k_page_scale", k_page_scale), ("v_page_scale", v_page_scale)):
        if (scale.device.type != "cuda" or scale.dtype != torch.float16
                or tuple(scale.shape) != (old_k_cache.shape[0], HKV) or not scale.is_contiguous()):
            raise ValueError(f"{name} must be contiguous CUDA [old_pages,{HKV}] float16")
    if (old_kv_len.device.type != "cuda" or old_kv_len.dtype != torch.int32
            or tuple(old_kv_len.shape) != (batch,) or not old_kv_len.is_contiguous()):
        raise ValueError("old_kv_len must be contiguous CUDA [B] int32")
    if bool(torch.any(old_kv_len % PAGE).item()):
        raise ValueError(f"old_kv_len must be page-aligned ({PAGE} tokens)")
    if (value_center.device.type != "cuda" or value_center.dtype != torch.float16
            or tuple(value_center.shape) != (batch, HKV, DIM) or not value_center.is_contiguous()):
        raise ValueError(f"value_center must be contiguous CUDA [B,{HKV},{DIM}] float16")


def run_decode(wrapper, query, old_k_cache, old_v_cache, k_page_scale, v_page_scale, exact_k_cache,
               exact_v_cache, old_kv_len, value_center, **run_kwargs):
    validate_run_inputs(query, old_k_cache, old_v_cache, k_page_scale, v_page_scale, exact_k_cache,
                        exact_v_cache, old_kv_len, value_center)
    return wrapper.run(query, (old_k_cache, old_v_cache), k_page_scale, v_page_scale, exact_k_cache,
                       exact_v_cache, old_kv_len, value_center, 1.0 / math.sqrt(DIM), **run_kwargs)


__all__ = ["DIM", "HKV", "HQ", "PAGE", "make_heterogeneous_page_gauge_wrapper", "plan_decode",
           "run_decode", "validate_run_inputs"]
