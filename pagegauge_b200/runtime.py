"""Drop-in replacement of the PageGauge append extension module.

``load_append_extension()`` mirrors scripts/page_gauge_runtime.py:16-29 and
returns an object exposing the five operators of the reference's pybind
module (tests/page_gauge_append_extension.cu:1030-1041) with the same
argument order, the same in-place semantics and the same RuntimeError
messages for invalid arguments (:23-40, :585-640, :747-1011).  The work is
done by the sm_100a kernels of libpagegauge_b200.so on the current torch
CUDA stream; nothing is allocated on the device.
"""

from __future__ import annotations

import torch

from . import _lib

HEAD_DIM = 128
PAGE = 16


def _stream(tensor: torch.Tensor) -> int:
    return torch.cuda.current_stream(tensor.device).cuda_stream


def check_tensor(tensor: torch.Tensor, name: str, dtype: torch.dtype, dims: int) -> None:
    """tests/page_gauge_append_extension.cu:23-32."""
    if not tensor.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if tensor.dtype != dtype:
        raise RuntimeError(f"{name} has the wrong dtype")
    if tensor.dim() != dims:
        raise RuntimeError(f"{name} has the wrong rank")
    if not tensor.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def check_head_major_input(tensor: torch.Tensor, name: str) -> None:
    """tests/page_gauge_append_extension.cu:34-40."""
    if not tensor.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if tensor.dtype != torch.float16:
        raise RuntimeError(f"{name} must be FP16")
    if tensor.dim() != 3:
        raise RuntimeError(f"{name} must have rank three")
    if tensor.stride(2) != 1 or tensor.stride(1) != HEAD_DIM:
        raise RuntimeError(f"{name} must be head-major with a contiguous head dimension")


def _require(cond: bool, message: str) -> None:
    if not cond:
        raise RuntimeError(message)


def _check_qkv(query, key, value, rotated_query) -> None:
    check_head_major_input(query, "query")
    check_head_major_input(key, "key")
    check_head_major_input(value, "value")
    check_tensor(rotated_query, "rotated_query", torch.float16, 3)
    _require(query.size(0) > 0 and query.size(0) == key.size(0) and query.size(0) == value.size(0),
             "Q/K/V batch sizes must match and be positive")
    _require(query.size(2) == HEAD_DIM and key.size(2) == HEAD_DIM and value.size(2) == HEAD_DIM,
             "head dimension must be 128")
    _require(key.shape == value.shape, "K/V input shapes must match")
    _require(rotated_query.shape == query.shape, "rotated query shape mismatch")


def _check_host_or_device_input(tensor, name: str) -> None:
    """A head-major FP16 input that may also be page-locked host memory."""
    if not (tensor.is_cuda or tensor.is_pinned()):
        raise RuntimeError(f"{name} must be CUDA or page-locked host memory")
    if tensor.dtype != torch.float16:
        raise RuntimeError(f"{name} must be FP16")
    if tensor.dim() != 3:
        raise RuntimeError(f"{name} must have rank three")
    if tensor.stride(2) != 1 or tensor.stride(1) != HEAD_DIM:
        raise RuntimeError(f"{name} must be head-major with a contiguous head dimension")


def _check_dynamic(query, cosine, sine, position) -> None:
    """tests/page_gauge_append_extension.cu:623-640."""
    check_tensor(cosine, "cosine", torch.float16, 2)
    check_tensor(sine, "sine", torch.float16, 2)
    check_tensor(position, "position", torch.int32, 1)
    _require(cosine.shape == sine.shape and cosine.size(0) > 0 and cosine.size(1) == HEAD_DIM,
             "dynamic RoPE tables must be matching [positions,128] tensors")
    _require(position.numel() == 1, "dynamic position must contain exactly one int32 scalar")
    _require(cosine.device == query.device and sine.device == query.device
             and position.device == query.device,
             "dynamic position, RoPE tables, and Q/K/V must share one device")


def _check_positions(query, cosine, sine, positions) -> None:
    """Per-request positions: device int32 [B] plus [positions,128] tables."""
    check_tensor(cosine, "cosine", torch.float16, 2)
    check_tensor(sine, "sine", torch.float16, 2)
    check_tensor(positions, "positions", torch.int32, 1)
    _require(cosine.shape == sine.shape and cosine.size(0) > 0 and cosine.size(1) == HEAD_DIM,
             "dynamic RoPE tables must be matching [positions,128] tensors")
    _require(positions.numel() == query.size(0), "positions must hold one int32 per request")
    _require(cosine.device == query.device and sine.device == query.device
             and positions.device == query.device,
             "dynamic position, RoPE tables, and Q/K/V must share one device")


def _check_pages(pages_k, pages_v, key, name_k, name_v, message) -> None:
    check_tensor(pages_k, name_k, torch.float16, 4)
    check_tensor(pages_v, name_v, torch.float16, 4)
    _require(pages_k.shape == pages_v.shape and pages_k.size(1) == PAGE
             and pages_k.size(2) == key.size(1) and pages_k.size(3) == HEAD_DIM, message)


def _check_gauge_storage(query, key, key_center, value_center, key_codes, value_codes,
                         key_scales, value_scales) -> int:
    """Centre/code/scale checks of tests/page_gauge_append_extension.cu:766-813.
    Returns the centre batch stride in elements (0 for a shared centre)."""
    _require(key_center.is_cuda and value_center.is_cuda, "centers must be CUDA")
    _require(key_center.dtype == torch.float16 and value_center.dtype == torch.float16,
             "centers must be FP16")
    _require(key_center.is_contiguous() and value_center.is_contiguous(), "centers must be contiguous")
    check_tensor(key_codes, "key_codes", torch.int8, 4)
    check_tensor(value_codes, "value_codes", torch.int8, 4)
    check_tensor(key_scales, "key_scales", torch.float16, 2)
    check_tensor(value_scales, "value_scales", torch.float16, 2)
    kv_heads = key.size(1)
    batch = query.size(0)
    ok = key_center.shape == value_center.shape and (
        (batch == 1 and key_center.dim() == 2 and key_center.size(0) == kv_heads
         and key_center.size(1) == HEAD_DIM)
        or (key_center.dim() == 3 and key_center.size(0) == batch
            and key_center.size(1) == kv_heads and key_center.size(2) == HEAD_DIM))
    _require(ok, "centers must be [B,Hkv,128] (or [Hkv,128] for batch one)")
    _require(key_codes.shape == value_codes.shape and key_codes.size(1) == PAGE
             and key_codes.size(2) == kv_heads and key_codes.size(3) == HEAD_DIM,
             "INT8 caches must be NHD [pages,16,Hkv,128]")
    _require(key_scales.shape == value_scales.shape and key_scales.size(0) == key_codes.size(0)
             and key_scales.size(1) == kv_heads, "scales must be [pages,Hkv]")
    return 0 if key_center.dim() == 2 else kv_heads * HEAD_DIM


class AppendExtension:
    """Operator table of the reference append extension."""

    def rope_append_fp16(self, query, key, value, cosine, sine, rotated_query,
                         key_pages, value_pages, position: int) -> None:
        _check_qkv(query, key, value, rotated_query)
        check_tensor(cosine, "cosine", torch.float16, 1)
        check_tensor(sine, "sine", torch.float16, 1)
        _check_pages(key_pages, value_pages, key, "key_pages", "value_pages",
                     "page cache must be NHD [pages,16,Hkv,128]")
        _require(cosine.numel() == HEAD_DIM and sine.numel() == HEAD_DIM,
                 "RoPE vectors must contain 128 values")
        _require(position >= 0, "position must be non-negative")
        _lib.call(
            "pg_rope_append_fp16", query.data_ptr(), key.data_ptr(), value.data_ptr(),
            cosine.data_ptr(), sine.data_ptr(), rotated_query.data_ptr(), key_pages.data_ptr(),
            value_pages.data_ptr(), query.stride(0), key.stride(0), value.stride(0),
            query.size(0), query.size(1), key.size(1), key_pages.size(0), int(position),
            None, 0, 0, _stream(query))

    def rope_append_fp16_dynamic(self, query, key, value, cosine, sine, position,
                                 rotated_query, key_pages, value_pages) -> None:
        _check_qkv(query, key, value, rotated_query)
        check_tensor(key_pages, "key_pages", torch.float16, 4)
        check_tensor(value_pages, "value_pages", torch.float16, 4)
        _require(key_pages.shape == value_pages.shape and key_pages.size(1) == PAGE
                 and key_pages.size(2) == key.size(1) and key_pages.size(3) == HEAD_DIM,
                 "page cache must be NHD [pages,16,Hkv,128]")
        _check_dynamic(query, cosine, sine, position)
        _lib.call(
            "pg_rope_append_fp16", query.data_ptr(), key.data_ptr(), value.data_ptr(),
            cosine.data_ptr(), sine.data_ptr(), rotated_query.data_ptr(), key_pages.data_ptr(),
            value_pages.data_ptr(), query.stride(0), key.stride(0), value.stride(0),
            query.size(0), query.size(1), key.size(1), key_pages.size(0), 0,
            position.data_ptr(), cosine.stride(0), cosine.size(0), _stream(query))

    def rope_append_page_gauge(self, query, key, value, cosine, sine, key_center, value_center,
                               rotated_query, exact_key_pages, exact_value_pages, key_codes,
                               value_codes, key_scales, value_scales, exact_sink_pages: int,
                               position: int) -> None:
        _check_qkv(query, key, value, rotated_query)
        check_tensor(cosine, "cosine", torch.float16, 1)
        check_tensor(sine, "sine", torch.float16, 1)
        _check_pages(exact_key_pages, exact_value_pages, key, "key_pages", "value_pages",
                     "page cache must be NHD [pages,16,Hkv,128]")
        _require(cosine.numel() == HEAD_DIM and sine.numel() == HEAD_DIM,
                 "RoPE vectors must contain 128 values")
        _require(position >= 0, "position must be non-negative")
        cstride = _check_gauge_storage(query, key, key_center, value_center, key_codes,
                                       value_codes, key_scales, value_scales)
        self._gauge_call(query, key, value, cosine, sine, key_center, value_center,
                         rotated_query, exact_key_pages, exact_value_pages, key_codes,
                         value_codes, key_scales, value_scales, cstride, exact_sink_pages,
                         int(position), None, 0, 0)

    def rope_append_page_gauge_dynamic(self, query, key, value, cosine, sine, position,
                                       key_center, value_center, rotated_query, exact_key_pages,
                                       exact_value_pages, key_codes, value_codes, key_scales,
                                       value_scales, exact_sink_pages: int) -> None:
        check_head_major_input(query, "query")
        check_head_major_input(key, "key")
        check_head_major_input(value, "value")
        check_tensor(rotated_query, "rotated_query", torch.float16, 3)
        check_tensor(exact_key_pages, "exact_key_pages", torch.float16, 4)
        check_tensor(exact_value_pages, "exact_value_pages", torch.float16, 4)
        _require(query.size(0) > 0 and query.size(0) == key.size(0) and query.size(0) == value.size(0),
                 "Q/K/V batch sizes must match and be positive")
        _require(query.size(2) == HEAD_DIM and key.size(2) == HEAD_DIM and value.size(2) == HEAD_DIM,
                 "head dimension must be 128")
        _require(key.shape == value.shape, "K/V input shapes must match")
        _require(rotated_query.shape == query.shape, "rotated query shape mismatch")
        _require(exact_key_pages.shape == exact_value_pages.shape and exact_key_pages.size(1) == PAGE
                 and exact_key_pages.size(2) == key.size(1) and exact_key_pages.size(3) == HEAD_DIM,
                 "exact page cache must be NHD [pages,16,Hkv,128]")
        _check_dynamic(query, cosine, sine, position)
        cstride = _check_gauge_storage(query, key, key_center, value_center, key_codes,
                                       value_codes, key_scales, value_scales)
        self._gauge_call(query, key, value, cosine, sine, key_center, value_center,
                         rotated_query, exact_key_pages, exact_value_pages, key_codes,
                         value_codes, key_scales, value_scales, cstride, exact_sink_pages, 0,
                         position.data_ptr(), cosine.stride(0), cosine.size(0))

    def rope_append_fp16_batched(self, query, key, value, cosine, sine, positions,
                                 rotated_query, key_pages, value_pages) -> None:
        """rope_append_fp16_dynamic with one position per request
        (``positions`` int32 [B] on the device)."""
        _check_qkv(query, key, value, rotated_query)
        _check_pages(key_pages, value_pages, key, "key_pages", "value_pages",
                     "page cache must be NHD [pages,16,Hkv,128]")
        _check_positions(query, cosine, sine, positions)
        _lib.call(
            "pg_rope_append_fp16_batched", query.data_ptr(), key.data_ptr(), value.data_ptr(),
            cosine.data_ptr(), sine.data_ptr(), rotated_query.data_ptr(), key_pages.data_ptr(),
            value_pages.data_ptr(), query.stride(0), key.stride(0), value.stride(0),
            query.size(0), query.size(1), key.size(1), key_pages.size(0),
            positions.data_ptr(), cosine.stride(0), cosine.size(0), _stream(query))

    def rope_append_page_gauge_batched(self, query, key, value, cosine, sine, positions,
                                       key_center, value_center, rotated_query, exact_key_pages,
                                       exact_value_pages, key_codes, value_codes, key_scales,
                                       value_scales, exact_sink_pages: int,
                                       inputs_ready: bool = False) -> None:
        """rope_append_page_gauge_dynamic with one position per request
        (``positions`` int32 [B] on the device): request r appends at
        positions[r] and closes its page when positions[r] % 16 == 15.
        ``query``/``key``/``value`` may be page-locked host tensors: the
        kernel then reads them over the host link (no separate copy).
        ``inputs_ready=True`` declares that no kernel earlier in the stream
        writes query/key/value (host rows written before the call): the
        kernel requests them before waiting for the previous kernel."""
        host_in = not query.is_cuda
        if host_in:
            for name, t in (("query", query), ("key", key), ("value", value)):
                _check_host_or_device_input(t, name)
            check_tensor(rotated_query, "rotated_query", torch.float16, 3)
            _require(query.size(0) > 0 and query.size(0) == key.size(0)
                     and query.size(0) == value.size(0),
                     "Q/K/V batch sizes must match and be positive")
            _require(key.shape == value.shape, "K/V input shapes must match")
            _require(rotated_query.shape == query.shape, "rotated query shape mismatch")
            _check_positions(rotated_query, cosine, sine, positions)
        else:
            _check_qkv(query, key, value, rotated_query)
            _check_positions(query, cosine, sine, positions)
        _check_pages(exact_key_pages, exact_value_pages, key, "exact_key_pages",
                     "exact_value_pages", "exact page cache must be NHD [pages,16,Hkv,128]")
        cstride = _check_gauge_storage(query, key, key_center, value_center, key_codes,
                                       value_codes, key_scales, value_scales)
        _lib.call(
            "pg_rope_append_page_gauge_batched", _lib.kernel_pointer(query, "query"),
            _lib.kernel_pointer(key, "key"), _lib.kernel_pointer(value, "value"),
            cosine.data_ptr(), sine.data_ptr(), key_center.data_ptr(),
            value_center.data_ptr(), rotated_query.data_ptr(), exact_key_pages.data_ptr(),
            exact_value_pages.data_ptr(), key_codes.data_ptr(), value_codes.data_ptr(),
            key_scales.data_ptr(), value_scales.data_ptr(), query.stride(0), key.stride(0),
            value.stride(0), cstride, query.size(0), query.size(1), key.size(1),
            exact_key_pages.size(0), key_codes.size(0), int(exact_sink_pages),
            positions.data_ptr(), cosine.stride(0), cosine.size(0), int(bool(inputs_ready)),
            _stream(rotated_query))

    def _gauge_call(self, query, key, value, cosine, sine, key_center, value_center,
                    rotated_query, exact_k, exact_v, codes_k, codes_v, scales_k, scales_v,
                    cstride, sink, position, device_position, rope_stride, rope_rows) -> None:
        _lib.call(
            "pg_rope_append_page_gauge", query.data_ptr(), key.data_ptr(), value.data_ptr(),
            cosine.data_ptr(), sine.data_ptr(), key_center.data_ptr(), value_center.data_ptr(),
            rotated_query.data_ptr(), exact_k.data_ptr(), exact_v.data_ptr(), codes_k.data_ptr(),
            codes_v.data_ptr(), scales_k.data_ptr(), scales_v.data_ptr(), query.stride(0),
            key.stride(0), value.stride(0), cstride, query.size(0), query.size(1), key.size(1),
            exact_k.size(0), codes_k.size(0), int(sink), position, device_position,
            rope_stride, rope_rows, _stream(query))

    def exact_tail_merge_center(self, query, exact_key_pages, exact_value_pages,
                                exact_page_indices, exact_last_page_len, old_output, old_lse,
                                value_center, sm_scale: float) -> None:
        """tests/page_gauge_append_extension.cu:950-1028 (checks kept)."""
        check_tensor(query, "query", torch.float16, 3)
        check_tensor(exact_key_pages, "exact_key_pages", torch.float16, 4)
        check_tensor(exact_value_pages, "exact_value_pages", torch.float16, 4)
        check_tensor(exact_page_indices, "exact_page_indices", torch.int32, 1)
        check_tensor(exact_last_page_len, "exact_last_page_len", torch.int32, 1)
        check_tensor(old_output, "old_output", torch.float16, 3)
        check_tensor(old_lse, "old_lse", torch.float32, 2)
        _require(value_center.is_cuda and value_center.dtype == torch.float16
                 and value_center.is_contiguous(), "value_center must be contiguous CUDA FP16")
        _require(query.shape == old_output.shape, "query and old output shapes must match")
        _require(query.size(2) == HEAD_DIM, "head dimension must be 128")
        _require(exact_key_pages.shape == exact_value_pages.shape and exact_key_pages.size(1) == PAGE
                 and exact_key_pages.size(3) == HEAD_DIM,
                 "exact caches must be matching NHD [pages,16,Hkv,128] tensors")
        batch, query_heads = query.size(0), query.size(1)
        _require(batch > 0, "batch size must be positive")
        kv_heads = exact_key_pages.size(2)
        _require(query_heads > 0 and kv_heads > 0 and query_heads % kv_heads == 0,
                 "query heads must be a positive multiple of KV heads")
        _require(old_lse.size(0) == batch and old_lse.size(1) == query_heads, "old_lse must be [B,Hq]")
        ok = ((batch == 1 and value_center.dim() == 2 and value_center.size(0) == kv_heads
               and value_center.size(1) == HEAD_DIM)
              or (value_center.dim() == 3 and value_center.size(0) == batch
                  and value_center.size(1) == kv_heads and value_center.size(2) == HEAD_DIM))
        _require(ok, "value_center must be [B,Hkv,128] (or [Hkv,128] for batch one)")
        _require(exact_last_page_len.numel() == batch,
                 "exact_last_page_len must contain one device scalar per request")
        cstride = 0 if value_center.dim() == 2 else kv_heads * HEAD_DIM
        _lib.call(
            "pg_exact_tail_merge_center", query.data_ptr(), exact_key_pages.data_ptr(),
            exact_value_pages.data_ptr(), exact_key_pages.size(0), exact_page_indices.data_ptr(),
            exact_page_indices.numel(), exact_last_page_len.data_ptr(), old_output.data_ptr(),
            old_lse.data_ptr(), value_center.data_ptr(), cstride, batch, query_heads, kv_heads,
            float(sm_scale), _stream(query))


_EXTENSION: AppendExtension | None = None


def load_append_extension() -> AppendExtension:
    """scripts/page_gauge_runtime.py:16-29: CUDA is required; the compiled
    sm_100a library must be present (no JIT build, no fallback)."""
    global _EXTENSION
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for the PageGauge append extension")
    _lib.load()
    if _EXTENSION is None:
        _EXTENSION = AppendExtension()
    return _EXTENSION


def read_device_error() -> int:
    """Read and clear the device guard word (0 = no guard fired)."""
    code = _lib.ctypes.c_int32(0)
    _lib.check(_lib.load().pg_read_device_error(_lib.ctypes.byref(code)))
    return int(code.value)
