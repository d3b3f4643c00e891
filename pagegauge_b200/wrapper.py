"""Paged decode wrappers with the FlashInfer ``plan``/``run`` surface the
PageGauge reference drives, backed by the sm_100a split-KV kernels.

* ``make_page_gauge_wrapper(flashinfer, workspace, **kw)`` replaces
  scripts/benchmark_flashinfer_page_affine_int8.py:192-231: INT8 codes with
  one FP16 scale per (page, KV head); ``run(q, (k_codes, v_codes), k_scale,
  v_scale, sm_scale, out=, lse=, return_lse=)`` returns the *centred*
  partial output and its base-2 log-sum-exp (c_V is not added), as the
  patched FA2 kernel does.
* ``make_affine_wrapper(flashinfer, workspace)`` replaces :166-189, the
  "affine_group16" representation: INT8 codes with an FP16 scale and bias
  per (page, KV head, 16-dim group); ``run(q, (k_codes, v_codes), k_bias,
  k_scale, v_bias, v_scale, sm_scale, out=, lse=, return_lse=)``.
* ``BatchDecodeWithPagedKVCacheWrapper(workspace, "NHD", ...)`` is the FP16
  paged decode used for the exact tail segment and the FP16 baseline.
* ``plan(wrapper, indptr, indices, last_page_len, kv_dtype, fixed_split_pages)``
  is the reference helper (:363-389).
* ``merge_state_in_place(v_a, s_a, v_b, s_b)`` merges two base-2 states.

The caller owns every buffer: work items and split partials are carved
from the workspace passed at construction, and in CUDA-graph mode the page
table buffers passed at construction are the ones the kernels read.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib

HEAD_DIM = 128
PAGE = 16
ITEM_BYTES = ctypes.sizeof(_lib.PgDecodeItem)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def num_sms(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def host_indptr(indptr) -> np.ndarray:
    """A host int32 copy of a CSR indptr given as a tensor or an array."""
    if isinstance(indptr, np.ndarray):
        return indptr.astype(np.int32, copy=True)
    return indptr.detach().to("cpu", torch.int32).numpy().astype(np.int32, copy=True)


def plan_items(batch: int, kv_heads: int, indptr0: np.ndarray | None,
               indptr1: np.ndarray | None, split0: int, split1: int, sms: int,
               warps: int = 4):
    """Run the host planner; returns (items bytes ndarray, item_off, info)."""
    lib = _lib.load()
    info = _lib.PgPlanInfo()
    off = np.zeros(batch * kv_heads + 1, dtype=np.int32)
    p0 = None if indptr0 is None else indptr0.ctypes.data
    p1 = None if indptr1 is None else indptr1.ctypes.data
    rc = lib.pg_decode_plan(batch, kv_heads, p0, p1, split0, split1, sms, warps, None, 0,
                            off.ctypes.data, ctypes.byref(info))
    if rc not in (0, 3):  # 3: capacity (sizing pass)
        _lib.check(rc)
    n = int(info.num_items)
    items = np.zeros((max(n, 1), 4), dtype=np.int32)
    _lib.check(lib.pg_decode_plan(batch, kv_heads, p0, p1, split0, split1, sms, warps,
                                  items.ctypes.data, n, off.ctypes.data, ctypes.byref(info)))
    return items[:n], off, info


class _Workspace:
    """Carves items / offsets / partial states out of the caller's buffer."""

    def __init__(self, buffer: torch.Tensor):
        if not buffer.is_cuda or buffer.dtype != torch.uint8 or not buffer.is_contiguous():
            raise ValueError("workspace must be a contiguous CUDA uint8 tensor")
        self.buffer = buffer

    def layout(self, num_items: int, num_offsets: int, group: int):
        def align(x: int) -> int:
            return (x + 255) // 256 * 256

        items_b = align(max(num_items, 1) * ITEM_BYTES)
        off_b = align(num_offsets * 4)
        sem_b = align(num_offsets * 4)
        lse_b = align(max(num_items, 1) * group * 4)
        o_b = align(max(num_items, 1) * group * HEAD_DIM * 4)
        total = items_b + off_b + sem_b + lse_b + o_b
        if total > self.buffer.numel():
            raise RuntimeError(
                f"workspace of {self.buffer.numel()} bytes is too small for {num_items} work items "
                f"({total} bytes needed); use a larger fixed_split_size")
        base = self.buffer
        items = base[:items_b]
        off = base[items_b:items_b + off_b]
        sem = base[items_b + off_b:items_b + off_b + sem_b]
        lse = base[items_b + off_b + sem_b:items_b + off_b + sem_b + lse_b]
        part_o = base[items_b + off_b + sem_b + lse_b:total]
        return items, off, sem, lse, part_o


class PagedDecodePlan:
    """Device-resident work list of one plan."""

    def __init__(self, ws: _Workspace, items: np.ndarray, off: np.ndarray, info, batch: int,
                 kv_heads: int, group: int):
        self.num_items = int(info.num_items)
        self.single = bool(info.single_item_per_head)
        self.split_pages = (int(info.split_pages[0]), int(info.split_pages[1]))
        self.warps = int(info.warps_per_cta)
        self.batch, self.kv_heads, self.group = batch, kv_heads, group
        d_items, d_off, d_sem, d_lse, d_o = ws.layout(self.num_items, off.size, group)
        d_sem.zero_()  # per-head arrival counters of the fused merge
        if self.num_items:
            src = torch.from_numpy(items.view(np.uint8).reshape(-1))
            d_items[:src.numel()].copy_(src, non_blocking=False)
        d_off[:off.size * 4].copy_(torch.from_numpy(off.view(np.uint8)), non_blocking=False)
        self.items_ptr = d_items.data_ptr()
        self.off_ptr = d_off.data_ptr()
        self.sem_ptr = d_sem.data_ptr()
        self.lse_ptr = d_lse.data_ptr()
        self.o_ptr = d_o.data_ptr()
        self.host_items = items
        self.host_off = off


def _segment(k, v, indices, last_len, k_scale=None, v_scale=None) -> _lib.PgSegment:
    seg = _lib.PgSegment()
    seg.k_cache = k.data_ptr()
    seg.v_cache = v.data_ptr()
    seg.num_pages = k.size(0)
    seg.indices = indices.data_ptr()
    seg.last_page_len = last_len.data_ptr()
    seg.k_scale = None if k_scale is None else k_scale.data_ptr()
    seg.v_scale = None if v_scale is None else v_scale.data_ptr()
    return seg


def check_cache(cache: torch.Tensor, name: str, dtype: torch.dtype, kv_heads: int) -> None:
    if (not cache.is_cuda or cache.dtype != dtype or cache.dim() != 4
            or tuple(cache.shape[1:]) != (PAGE, kv_heads, HEAD_DIM) or not cache.is_contiguous()):
        raise ValueError(f"{name} must be contiguous CUDA [pages,{PAGE},{kv_heads},{HEAD_DIM}] {dtype}")


def launch_decode(plan: PagedDecodePlan, q: torch.Tensor, segments, sm_scale: float,
                  out: torch.Tensor, lse: torch.Tensor | None, extra=None,
                  value_center: torch.Tensor | None = None, final_ok: bool = True,
                  fused_merge: bool = False, cluster: int = 0,
                  affine_bias=None, int8_after_wait: bool = False) -> "_lib.PgDecodeArgs":
    """Fill the C argument block and launch split decode (+ merge); returns
    the argument block so a caller may relaunch it unchanged.
    ``int8_after_wait``: the INT8 pages may have been written by a kernel
    launched just before (an append that closed a page of a one-page exact
    ring), so the decode reads them only after that kernel completes."""
    if q.dtype != torch.float16 or q.dim() != 3 or q.stride(2) != 1:
        raise ValueError("q must be float16 [B,Hq,128] with a contiguous last dimension")
    a = _lib.PgDecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
    a.batch, a.kv_heads, a.group = plan.batch, plan.kv_heads, plan.group
    a.sm_scale = float(sm_scale)
    for s, seg in enumerate(segments):
        if seg is not None:
            a.seg[s] = seg
    a.items = plan.items_ptr
    a.item_off = plan.off_ptr
    a.num_items = plan.num_items
    a.warps_per_cta = plan.warps
    a.part_o = plan.o_ptr
    a.part_lse = plan.lse_ptr
    a.final_mode = 1 if (final_ok and plan.single and plan.num_items > 0) else 0
    # One launch: the last CTA of a head merges it (fused_merge), or CTAs in
    # clusters of `cluster` work items merge through distributed shared
    # memory and the last cluster of a head finishes it.
    a.merge_sem = plan.sem_ptr if (fused_merge or cluster > 1) else None
    a.cluster = cluster
    # out / lse may be page-locked host tensors: the merge (or the final
    # epilogue) then writes the result over the host link.
    a.out = _lib.kernel_pointer(out, "out")
    a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
    a.lse_out = None if lse is None else _lib.kernel_pointer(lse, "lse")
    if extra is not None:
        eo, el = extra
        a.extra_o = eo.data_ptr()
        a.extra_stride_b, a.extra_stride_h = eo.stride(0), eo.stride(1)
        a.extra_lse = el.data_ptr()
    if value_center is not None:
        a.value_center = value_center.data_ptr()
        a.vc_stride_b = 0 if value_center.dim() == 2 else value_center.stride(0)
    if affine_bias is not None:
        # affine_group16: segment 0's scales are per 16-dim group, and these
        # are the matching biases.
        a.representation = 1
        a.k_bias = affine_bias[0].data_ptr()
        a.v_bias = affine_bias[1].data_ptr()
    a.int8_after_wait = 1 if int8_after_wait else 0
    _lib.check(_lib.load().pg_decode_run(ctypes.byref(a), _stream(q)))
    return a


class BatchDecodeWithPagedKVCacheWrapper:
    """FlashInfer-shaped paged decode wrapper (NHD, page 16, head_dim 128).

    ``page_gauge=True`` selects INT8 codes with per-(page, head) FP16 scales;
    ``affine_group16=True`` INT8 codes with an FP16 scale and bias per
    (page, head, 16-dim group).
    """

    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, use_tensor_cores: bool = True,
                 paged_kv_indptr_buffer: torch.Tensor | None = None,
                 paged_kv_indices_buffer: torch.Tensor | None = None,
                 paged_kv_last_page_len_buffer: torch.Tensor | None = None,
                 backend: str = "auto", jit_args=None, page_gauge: bool = False,
                 affine_group16: bool = False, **_ignored):
        if kv_layout != "NHD":
            raise ValueError("only the NHD page layout is supported")
        self._ws = _Workspace(float_workspace_buffer)
        self._use_cuda_graph = bool(use_cuda_graph)
        if self._use_cuda_graph and (paged_kv_indptr_buffer is None or paged_kv_indices_buffer is None
                                     or paged_kv_last_page_len_buffer is None):
            raise ValueError("use_cuda_graph requires indptr, indices and last_page_len buffers")
        self._paged_kv_indptr_buf = paged_kv_indptr_buffer
        self._paged_kv_indices_buf = paged_kv_indices_buffer
        self._paged_kv_last_page_len_buf = paged_kv_last_page_len_buffer
        if page_gauge and affine_group16:
            raise ValueError("choose one INT8 representation")
        self.affine_group16 = bool(affine_group16)
        self.page_gauge = bool(page_gauge) or self.affine_group16  # INT8 segment
        self._plan: PagedDecodePlan | None = None
        self._indices: torch.Tensor | None = None
        self._last_len: torch.Tensor | None = None
        self._sm_scale = 1.0 / math.sqrt(HEAD_DIM)
        self._kv_dtype = torch.int8 if self.page_gauge else torch.float16
        self.plan_invocations = 0

    @property
    def kv_data_type(self) -> torch.dtype:
        return self._kv_dtype

    def plan(self, indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             pos_encoding_mode: str = "NONE", window_left: int = -1, logits_soft_cap=None,
             q_data_type=torch.float16, kv_data_type=None, o_data_type=torch.float16,
             data_type=None, sm_scale: float | None = None, rope_scale=None, rope_theta=None,
             non_blocking: bool = True, fixed_split_size: int | None = None,
             disable_split_kv: bool = False, **_ignored) -> None:
        """Host planning (outside CUDA-graph capture), as FlashInfer's plan."""
        if head_dim != HEAD_DIM or page_size != PAGE:
            raise ValueError("PageGauge decode supports head_dim 128 and page size 16")
        if pos_encoding_mode != "NONE":
            raise ValueError("only pos_encoding_mode='NONE' is supported (RoPE is fused into append)")
        if window_left not in (-1, None) or logits_soft_cap not in (None, 0, 0.0):
            raise ValueError("sliding windows and logit soft caps are not supported")
        if num_kv_heads <= 0 or num_qo_heads % num_kv_heads or not 1 <= num_qo_heads // num_kv_heads <= 8:
            raise ValueError("num_qo_heads must be a multiple (1..8) of num_kv_heads")
        kvd = kv_data_type if kv_data_type is not None else data_type
        if kvd is not None:
            want = torch.int8 if self.page_gauge else torch.float16
            if kvd != want:
                raise ValueError(f"this wrapper decodes {want} pages, got {kvd}")
        for name, t in (("indptr", indptr), ("indices", indices), ("last_page_len", last_page_len)):
            if t.dtype != torch.int32:
                raise ValueError(f"{name} must be int32")
        self.plan_invocations += 1
        batch = indptr.numel() - 1
        if batch <= 0 or last_page_len.numel() != batch:
            raise ValueError("indptr/last_page_len batch dimensions disagree")
        if sm_scale is not None:
            self._sm_scale = float(sm_scale)
        ind = host_indptr(indptr)
        if self._use_cuda_graph:
            nnz = int(ind[-1])
            self._paged_kv_indptr_buf[: batch + 1].copy_(indptr, non_blocking=True)
            if indices.data_ptr() != self._paged_kv_indices_buf.data_ptr():
                self._paged_kv_indices_buf[:nnz].copy_(indices[:nnz], non_blocking=True)
            if last_page_len.data_ptr() != self._paged_kv_last_page_len_buf.data_ptr():
                self._paged_kv_last_page_len_buf[:batch].copy_(last_page_len, non_blocking=True)
            dev_indices = self._paged_kv_indices_buf
            dev_last = self._paged_kv_last_page_len_buf
        else:
            dev_indices = indices if indices.is_cuda else indices.cuda()
            dev_last = last_page_len if last_page_len.is_cuda else last_page_len.cuda()
        split = int(fixed_split_size or 0)
        if disable_split_kv:
            split = 1 << 30
        sms = num_sms(self._ws.buffer.device)
        seg0 = ind if self.page_gauge else None
        seg1 = None if self.page_gauge else ind
        items, off, info = plan_items(batch, num_kv_heads, seg0, seg1,
                                      min(split, 1 << 30), min(split, 1 << 30), sms)
        self._plan = PagedDecodePlan(self._ws, items, off, info, batch, num_kv_heads,
                                     num_qo_heads // num_kv_heads)
        self._indices = dev_indices
        self._last_len = dev_last
        self._num_qo_heads = num_qo_heads
        self._num_kv_heads = num_kv_heads

    begin_forward = plan

    @property
    def split_pages(self) -> int:
        if self._plan is None:
            raise RuntimeError("plan() has not been called")
        return self._plan.split_pages[0 if self.page_gauge else 1]

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None,
            v_scale=None, out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
            return_lse: bool = False, **_ignored):
        if self._plan is None:
            raise RuntimeError("plan() must be called before run()")
        k_cache, v_cache = paged_kv_cache
        sm_scale = self._sm_scale
        k_page_scale = v_page_scale = None
        affine_bias = None
        if self.affine_group16:
            # make_affine_wrapper's run(q, kv, k_bias, k_scale, v_bias, v_scale, sm_scale)
            if len(args) < 4:
                raise ValueError("affine run needs k_bias, k_scale, v_bias and v_scale")
            k_bias, k_page_scale, v_bias, v_page_scale = args[:4]
            if len(args) >= 5:
                sm_scale = float(args[4])
            shape = (k_cache.size(0), self._num_kv_heads, HEAD_DIM // 16)
            for name, t in (("k_bias", k_bias), ("k_scale", k_page_scale), ("v_bias", v_bias),
                            ("v_scale", v_page_scale)):
                if (not t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous()
                        or tuple(t.shape) != shape or t.data_ptr() % 16):
                    raise ValueError(f"{name} must be contiguous 16-byte aligned CUDA "
                                     f"[pages,{self._num_kv_heads},8] float16")
            affine_bias = (k_bias, v_bias)
        elif self.page_gauge:
            if len(args) < 2:
                raise ValueError("page-gauge run needs k_page_scale and v_page_scale")
            k_page_scale, v_page_scale = args[0], args[1]
            if len(args) >= 3:
                sm_scale = float(args[2])
            for name, s in (("k_page_scale", k_page_scale), ("v_page_scale", v_page_scale)):
                if (not s.is_cuda or s.dtype != torch.float16 or not s.is_contiguous()
                        or tuple(s.shape) != (k_cache.size(0), self._num_kv_heads)):
                    raise ValueError(f"{name} must be contiguous CUDA [pages,{self._num_kv_heads}] float16")
        check_cache(k_cache, "k_cache", self._kv_dtype, self._num_kv_heads)
        check_cache(v_cache, "v_cache", self._kv_dtype, self._num_kv_heads)
        if k_cache.shape != v_cache.shape:
            raise ValueError("K/V cache shapes must match")
        batch = self._plan.batch
        if tuple(q.shape) != (batch, self._num_qo_heads, HEAD_DIM):
            raise ValueError(f"q must be [{batch},{self._num_qo_heads},{HEAD_DIM}]")
        if out is None:
            out = torch.empty_like(q)
        if lse is None and return_lse:
            lse = torch.empty(batch, self._num_qo_heads, device=q.device, dtype=torch.float32)
        seg = _segment(k_cache, v_cache, self._indices, self._last_len, k_page_scale, v_page_scale)
        segments = (seg, None) if self.page_gauge else (None, seg)
        launch_decode(self._plan, q, segments, sm_scale, out, lse, affine_bias=affine_bias)
        return (out, lse) if return_lse else out

    forward = run


def make_page_gauge_wrapper(flashinfer=None, workspace: torch.Tensor | None = None,
                            **wrapper_kwargs) -> BatchDecodeWithPagedKVCacheWrapper:
    """scripts/benchmark_flashinfer_page_affine_int8.py:192-231 (the
    ``flashinfer`` module argument is accepted and ignored)."""
    if workspace is None:
        raise ValueError("a CUDA uint8 workspace is required")
    wrapper_kwargs.pop("jit_args", None)
    wrapper = BatchDecodeWithPagedKVCacheWrapper(workspace, "NHD", page_gauge=True, **wrapper_kwargs)
    wrapper.page_gauge_module_uri = "pagegauge_b200.sm100a.page_affine_int8"
    return wrapper


def make_affine_wrapper(flashinfer=None, workspace: torch.Tensor | None = None,
                        **wrapper_kwargs) -> BatchDecodeWithPagedKVCacheWrapper:
    """scripts/benchmark_flashinfer_page_affine_int8.py:166-189: the
    affine_group16 decode (the ``flashinfer`` argument is ignored)."""
    if workspace is None:
        raise ValueError("a CUDA uint8 workspace is required")
    wrapper_kwargs.pop("jit_args", None)
    wrapper = BatchDecodeWithPagedKVCacheWrapper(workspace, "NHD", affine_group16=True,
                                                 **wrapper_kwargs)
    wrapper.page_gauge_module_uri = "pagegauge_b200.sm100a.page_affine_int8_group16"
    return wrapper


def plan(wrapper: BatchDecodeWithPagedKVCacheWrapper, indptr, indices, last_page_len, kv_dtype,
         fixed_split_pages: int = 0, num_qo_heads: int = 32, num_kv_heads: int = 8,
         head_dim: int = HEAD_DIM, page_size: int = PAGE) -> None:
    """scripts/benchmark_flashinfer_page_affine_int8.py:363-389."""
    wrapper.plan(indptr, indices, last_page_len, num_qo_heads, num_kv_heads, head_dim, page_size,
                 pos_encoding_mode="NONE", q_data_type=torch.float16, kv_data_type=kv_dtype,
                 o_data_type=torch.float16, sm_scale=1.0 / math.sqrt(head_dim),
                 fixed_split_size=fixed_split_pages or None)


def merge_state_in_place(v: torch.Tensor, s: torch.Tensor, v_other: torch.Tensor,
                         s_other: torch.Tensor, mask=None) -> None:
    """flashinfer.merge_state_in_place: (v, s) <- merge((v, s), (v_other, s_other))
    with base-2 log-sum-exp; v [rows.., 128] fp16, s [rows..] fp32."""
    if mask is not None:
        raise ValueError("masked merge is not supported")
    if v.dtype != torch.float16 or v_other.dtype != torch.float16:
        raise ValueError("states must be float16")
    if s.dtype != torch.float32 or s_other.dtype != torch.float32:
        raise ValueError("lse must be float32")
    if v.shape != v_other.shape or v.shape[:-1] != s.shape or s.shape != s_other.shape:
        raise ValueError("state shapes disagree")
    if v.shape[-1] != HEAD_DIM:
        raise ValueError("head dimension must be 128")
    if not (v.is_contiguous() and v_other.is_contiguous() and s.is_contiguous() and s_other.is_contiguous()):
        raise ValueError("states must be contiguous")
    rows = s.numel()
    _lib.check(_lib.load().pg_merge_state_in_place(
        v.data_ptr(), s.data_ptr(), v_other.data_ptr(), s_other.data_ptr(), rows, HEAD_DIM,
        HEAD_DIM, _stream(v)))
