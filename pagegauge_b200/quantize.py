"""Completed-page INT8 quantisation on the GPU.

* ``quantize_completed_kv_pages`` replaces the Triton prefill quantiser
  (scripts/benchmark_page_gauge_overheads.py:23-83, :208-239): fp32 centring,
  scale = f16(max(absmax/127, 2^-20)), half-away-from-zero codes.
* ``quantize_page_gauge`` reproduces the PyTorch representation function
  (scripts/benchmark_flashinfer_page_affine_int8.py:256-278): centre = FP16
  mean over all tokens, one scale per (page, head), torch.round (half to
  even) codes; it returns (codes, center, scale, reconstructed_centered,
  centered) like the reference.
"""

from __future__ import annotations

import torch

from . import _lib

PAGE = 16
DIM = 128


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def quantize_pages_into(key, value, key_center, value_center, key_codes, value_codes,
                        key_scales, value_scales, pages_per_center: int = 0,
                        rounding: str = "half_away") -> None:
    """Quantise [pages,16,Hkv,128] FP16 K/V into codes/scales in place.

    Centres are [Hkv,128] (one for all pages) or [C,Hkv,128] with
    ``pages_per_center`` consecutive pages per centre row."""
    for name, t in (("key", key), ("value", value)):
        if not t.is_cuda or t.dtype != torch.float16 or t.dim() != 4 or t.shape[1] != PAGE \
                or t.shape[3] != DIM or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous CUDA [pages,16,heads,128] float16")
    if key.shape != value.shape:
        raise ValueError("K and V must have identical [pages, 16, heads, 128] shapes")
    pages, _, heads, _ = key.shape
    for name, c in (("key_center", key_center), ("value_center", value_center)):
        if c.dtype != torch.float16 or not c.is_contiguous() or c.shape[-2:] != (heads, DIM):
            raise ValueError("centers must be [heads, 128]")
    for name, t in (("key_codes", key_codes), ("value_codes", value_codes)):
        if t.dtype != torch.int8 or t.shape != key.shape or not t.is_contiguous():
            raise ValueError(f"{name} must be int8 {tuple(key.shape)}")
    for name, t in (("key_scales", key_scales), ("value_scales", value_scales)):
        if t.dtype != torch.float16 or tuple(t.shape) != (pages, heads) or not t.is_contiguous():
            raise ValueError(f"{name} must be float16 [{pages},{heads}]")
    mode = {"half_away": 0, "half_even": 1}[rounding]
    _lib.call("pg_quantize_pages", key.data_ptr(), value.data_ptr(), key_center.data_ptr(),
              value_center.data_ptr(), int(pages_per_center), key_codes.data_ptr(),
              value_codes.data_ptr(), key_scales.data_ptr(), value_scales.data_ptr(), pages,
              heads, mode, _stream(key))


def quantize_completed_kv_pages(key, value, key_center, value_center, key_codes, value_codes,
                                key_scales, value_scales) -> None:
    """Signature of scripts/benchmark_page_gauge_overheads.py:208-239."""
    if key.shape != value.shape or key.ndim != 4:
        raise ValueError("K and V must have identical [pages, 16, heads, 128] shapes")
    if key.shape[1] != PAGE or key.shape[-1] != DIM:
        raise ValueError("K and V must have shape [pages, 16, heads, 128]")
    if key_center.shape != (key.shape[2], DIM) or value_center.shape != key_center.shape:
        raise ValueError("centers must be [heads, 128]")
    quantize_pages_into(key, value, key_center, value_center, key_codes, value_codes, key_scales,
                        value_scales, 0, "half_away")


def _quantize_one(values: torch.Tensor, center: torch.Tensor):
    """One tensor's pages: the bulk quantiser's key-only form, torch.round."""
    if not values.is_cuda or values.dtype != torch.float16 or not values.is_contiguous():
        raise ValueError("values must be contiguous CUDA [pages,16,heads,128] float16")
    codes = torch.empty_like(values, dtype=torch.int8)
    scale = torch.empty(values.shape[0], values.shape[2], device=values.device, dtype=torch.float16)
    _lib.call("pg_quantize_pages", values.data_ptr(), None, center.data_ptr(), None, 0,
              codes.data_ptr(), None, scale.data_ptr(), None, values.shape[0], values.shape[2],
              1, _stream(values))
    return codes, scale


def quantize_page_gauge(values: torch.Tensor):
    """Return (codes, center, scale, reconstructed_centered, centered)."""
    if values.ndim != 4 or values.shape[1:] != (PAGE, values.shape[2], DIM):
        raise ValueError("values must be [pages, 16, HKV, 128]")
    values = values.contiguous()
    center = values.float().mean(dim=(0, 1)).half().contiguous()
    codes, scale = _quantize_one(values, center)
    reconstructed = (codes.float() * scale.float()[:, None, :, None]).half()
    centered = (values.float() - center.float()[None, None]).half()
    return codes, center, scale, reconstructed, centered


def quantize_pages(values: torch.Tensor):
    """affine_group16 representation (scripts/benchmark_flashinfer_page_affine_int8.py:234-253),
    bit-exact: per (page, KV head, 16-dim group) an FP16 scale and bias,
    codes = round_half_even((x - min) / scale) - 128.  Returns (codes int8
    [pages,16,H,128], bias [pages,H,8], scale [pages,H,8], reconstructed
    FP16 [pages,16,H,128]) like the reference."""
    if values.ndim != 4 or values.shape[1] != PAGE or values.shape[3] != DIM:
        raise ValueError("values must be [pages, 16, HKV, 128]")
    if not values.is_cuda or values.dtype != torch.float16:
        raise ValueError("values must be a CUDA float16 tensor")
    values = values.contiguous()
    pages, _, heads, _ = values.shape
    codes = torch.empty(values.shape, device=values.device, dtype=torch.int8)
    bias = torch.empty(pages, heads, DIM // 16, device=values.device, dtype=torch.float16)
    scale = torch.empty_like(bias)
    recon = torch.empty_like(values)
    _lib.call("pg_quantize_affine_group16", values.data_ptr(), pages, heads, codes.data_ptr(),
              bias.data_ptr(), scale.data_ptr(), recon.data_ptr(), _stream(values))
    return codes, bias, scale, recon
