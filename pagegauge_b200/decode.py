"""Fused PageGauge decode attention: old INT8 pages + exact FP16 pages,
LSE merge and value-centre restore in one split-KV launch plus one merge
launch (or a single launch when every (request, KV head) fits one CTA).

This is the B200 form of the reference's segmented eager attention
(scripts/benchmark_page_gauge_transformer.py:2261-2308: old_wrapper.run +
exact_wrapper.run + merge_state_in_place + add_(output_center)) and of its
single-launch heterogeneous ABI (scripts/page_gauge_heterogeneous_fa2.py).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from .wrapper import (HEAD_DIM, PAGE, PagedDecodePlan, _segment, _stream, _Workspace,
                      check_cache, host_indptr, launch_decode, num_sms, plan_items)


class PageGaugeDecode:
    """Plan once per page-table change, run per layer/step (graph-safe)."""

    def __init__(self, workspace: torch.Tensor, warps_per_cta: int = 4):
        self._ws = _Workspace(workspace)
        self._warps = warps_per_cta
        self._plan: PagedDecodePlan | None = None
        self.sm_scale = 1.0 / math.sqrt(HEAD_DIM)
        # Argument block of the last launch and the tensors it was built
        # from: a run with identical tensors relaunches it without
        # re-validating (the per-layer decode loop calls run() with the
        # same buffers every step).
        self._last_key = None
        self._last_args = None

    def plan(self, old_indptr, old_indices, exact_indptr, exact_indices, exact_last_page_len,
             num_qo_heads: int = 32, num_kv_heads: int = 8, old_split_pages: int = 0,
             exact_split_pages: int = 0, old_last_page_len: torch.Tensor | None = None,
             sm_scale: float | None = None) -> None:
        """``*_indptr`` CSR over the per-request page ids (host or device);
        ``*_indices`` device int32.  Old pages are full unless
        ``old_last_page_len`` says otherwise."""
        if num_qo_heads % num_kv_heads or not 1 <= num_qo_heads // num_kv_heads <= 8:
            raise ValueError("num_qo_heads must be a multiple (1..8) of num_kv_heads")
        o_ind = None if old_indptr is None else host_indptr(old_indptr)
        e_ind = None if exact_indptr is None else host_indptr(exact_indptr)
        batch = (o_ind if o_ind is not None else e_ind).size - 1
        dev = self._ws.buffer.device
        items, off, info = plan_items(batch, num_kv_heads, o_ind, e_ind, int(old_split_pages),
                                      int(exact_split_pages), num_sms(dev), self._warps)
        self._plan = PagedDecodePlan(self._ws, items, off, info, batch, num_kv_heads,
                                     num_qo_heads // num_kv_heads)
        self._last_key = self._last_args = None
        self._old_indices = old_indices
        self._exact_indices = exact_indices
        self._exact_last = exact_last_page_len
        if old_last_page_len is None and o_ind is not None:
            old_last_page_len = torch.full((batch,), PAGE, dtype=torch.int32, device=dev)
        self._old_last = old_last_page_len
        self._num_qo_heads, self._num_kv_heads = num_qo_heads, num_kv_heads
        if sm_scale is not None:
            self.sm_scale = float(sm_scale)

    @property
    def work_plan(self) -> PagedDecodePlan:
        if self._plan is None:
            raise RuntimeError("plan() has not been called")
        return self._plan

    def run(self, q: torch.Tensor, key_codes, value_codes, key_scales, value_scales,
            exact_key, exact_value, value_center: torch.Tensor | None,
            out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
            sm_scale: float | None = None, fused_merge: bool = False,
            cluster: int = 0, affine_bias=None, int8_after_wait: bool = False) -> torch.Tensor:
        """``cluster`` = 2..8 runs the decode as one launch whose CTAs merge
        in thread-block clusters (the single-launch ABI of the reference's
        heterogeneous path); ``fused_merge`` merges in the last CTA of each
        head; otherwise a merge kernel follows the split kernel.
        ``affine_bias = (k_bias, v_bias)`` selects the affine_group16
        representation for the INT8 pages: key/value_scales and the biases
        are then [pages, Hkv, 8] (one pair per 16-dim group).
        ``int8_after_wait`` must be set when an append launched just before
        this decode may have closed a page that this decode reads as INT8 --
        a one-page exact ring, where the page closed at one step is INT8 at
        the next.  The INT8 tiles are then requested only after the previous
        kernel in the stream completes (otherwise they are requested while it
        drains, because every kernel here lets its successor start early)."""
        plan = self.work_plan
        key = None
        if out is not None:
            key = (q.data_ptr(), q.shape, q.stride(), key_codes.data_ptr(), key_codes.shape,
                   value_codes.data_ptr(), key_scales.data_ptr(), value_scales.data_ptr(),
                   None if exact_key is None else (exact_key.data_ptr(), exact_key.shape,
                                                   exact_value.data_ptr()),
                   None if value_center is None else (value_center.data_ptr(), value_center.shape),
                   out.data_ptr(), out.shape, out.stride(), None if lse is None else lse.data_ptr(),
                   sm_scale, fused_merge, cluster, q.dtype, out.dtype, int8_after_wait,
                   None if affine_bias is None else (affine_bias[0].data_ptr(),
                                                     affine_bias[1].data_ptr()))
            if key == self._last_key:
                _lib.check(_lib.load().pg_decode_run(self._last_args_ref, _stream(q)))
                return out
        segs = [None, None]
        if self._old_indices is not None:
            check_cache(key_codes, "key_codes", torch.int8, self._num_kv_heads)
            check_cache(value_codes, "value_codes", torch.int8, self._num_kv_heads)
            segs[0] = _segment(key_codes, value_codes, self._old_indices, self._old_last,
                               key_scales, value_scales)
        if self._exact_indices is not None:
            check_cache(exact_key, "exact_key", torch.float16, self._num_kv_heads)
            check_cache(exact_value, "exact_value", torch.float16, self._num_kv_heads)
            segs[1] = _segment(exact_key, exact_value, self._exact_indices, self._exact_last)
        if out is None:
            out = torch.empty_like(q)
        if value_center is not None and (value_center.dtype != torch.float16
                                         or not value_center.is_contiguous()):
            raise ValueError("value_center must be contiguous float16")
        if affine_bias is not None:
            shape = (key_codes.size(0), self._num_kv_heads, 8)
            for name, t in (("key_scales", key_scales), ("value_scales", value_scales),
                            ("k_bias", affine_bias[0]), ("v_bias", affine_bias[1])):
                if (t.dtype != torch.float16 or not t.is_contiguous() or tuple(t.shape) != shape
                        or t.data_ptr() % 16):
                    raise ValueError(f"{name} must be contiguous 16-byte aligned "
                                     f"[pages,{self._num_kv_heads},8] float16")
        args = launch_decode(plan, q, segs, self.sm_scale if sm_scale is None else sm_scale, out,
                             lse, value_center=value_center, fused_merge=fused_merge,
                             cluster=cluster, affine_bias=affine_bias,
                             int8_after_wait=int8_after_wait)
        if key is not None:
            self._last_key, self._last_args = key, args
            self._last_args_ref = ctypes.byref(args)
        return out


def split_tables(pages_per_row, exact_tail_pages: int, exact_sink_pages: int = 0):
    """Host CSR tables of the old INT8 segment and the exact segment for
    request-major contiguous storage (segment_page_table semantics,
    scripts/benchmark_flashinfer_page_affine_int8.py:392-420)."""
    old_counts = [max(c - exact_tail_pages - exact_sink_pages, 0) for c in pages_per_row]
    exact_counts = [c - o for c, o in zip(pages_per_row, old_counts)]
    old_idx, exact_idx = [], []
    start = 0
    for count, old in zip(pages_per_row, old_counts):
        mid = start + exact_sink_pages
        old_idx.extend(range(mid, mid + old))
        exact_idx.extend(range(start, mid))
        exact_idx.extend(range(mid + old, start + count))
        start += count
    def csr(counts):
        return np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return csr(old_counts), np.asarray(old_idx, np.int32), csr(exact_counts), np.asarray(exact_idx, np.int32)
