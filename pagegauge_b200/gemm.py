"""Weight-streaming projections of the decoder (the C ABI's
``pg_skinny_gemm``): ``y = x @ w.T`` for up to 32 token rows with the
decoder layer's element-wise step fused into the epilogue.

The reference runs these projections through cuBLAS (``F.linear`` in the
decoder layer, scripts/benchmark_page_gauge_transformer.py:2754-2804).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

STORE, RESIDUAL, SILU_MUL = 0, 1, 2


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class PackedWeight:
    """W [n, k] FP16 in the kernel's tiled layout (one contiguous 8 KB block
    per 64 rows x 64 k, 128-byte swizzled; in silu_mul mode each tile holds
    32 gate rows and the matching 32 up rows)."""

    def __init__(self, w: torch.Tensor, mode: int = STORE):
        if w.dtype != torch.float16 or w.dim() != 2 or not w.is_cuda or w.stride(1) != 1:
            raise ValueError("w must be a CUDA float16 [n, k] tensor with contiguous rows")
        self.n, self.k = w.shape
        self.mode = mode
        self.data = torch.empty(self.n * self.k, dtype=torch.float16, device=w.device)
        _lib.check(_lib.load().pg_pack_weight(w.data_ptr(), w.stride(0), self.n, self.k, mode,
                                              self.data.data_ptr(), _stream()))

    @property
    def shape(self):
        return (self.n, self.k)


class SkinnyGemm:
    """Launcher with caller-owned split-K scratch (partial tiles + per-tile
    arrival counters), sized for the largest shape it is asked to run."""

    def __init__(self, device, partial_floats: int = 1 << 20, counters: int = 1024):
        self.device = torch.device(device)
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.partials = torch.empty(partial_floats, dtype=torch.float32, device=self.device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)

    def reserve(self, n: int, k: int, batch: int, mode: int = STORE, grid: int = 0) -> None:
        """Grow the scratch for a shape launched with ``grid`` CTAs (0: the
        default, one per resident slot) (host-side; outside graph capture)."""
        floats, tiles = ctypes.c_int64(0), ctypes.c_int32(0)
        _lib.check(_lib.load().pg_skinny_gemm_workspace(n, k, batch, mode, grid, self.sms,
                                                        ctypes.byref(floats), ctypes.byref(tiles)))
        if floats.value > self.partials.numel():
            self.partials = torch.empty(floats.value, dtype=torch.float32, device=self.device)
        if tiles.value > self.counters.numel():
            self.counters = torch.zeros(tiles.value, dtype=torch.int32, device=self.device)

    def __call__(self, x: torch.Tensor, w: PackedWeight, out: torch.Tensor | None = None,
                 mode: int = STORE, residual: torch.Tensor | None = None, pdl: bool = True,
                 grid: int = 0, norm_weight: torch.Tensor | None = None,
                 eps: float = 1e-5, tp=None) -> torch.Tensor | None:
        """y = x @ W^T with W packed for this ``mode`` (silu_mul needs the
        silu_mul packing; store and residual share theirs).  ``norm_weight``
        ([k] float16) first RMS-normalises the rows of x inside the GEMM
        (transformers' MistralRMSNorm: f16(w * f16(x * rsqrt(mean(x^2) +
        eps)))).  ``tp`` (a ``peer.TpExchange``, store mode): this rank's
        product is a partial sum; every finished tile is published to every
        rank through peer memory and nothing is written here -- the next
        ``tp.reduce`` sums the ranks' tiles (the row-parallel projection and
        its all-reduce without a collective library)."""
        if x.dtype != torch.float16 or x.dim() != 2 or x.stride(1) != 1:
            raise ValueError("x must be a float16 [batch, k] tensor with contiguous rows")
        if (w.mode == SILU_MUL) != (mode == SILU_MUL):
            raise ValueError("the weight was packed for another epilogue")
        batch, k = x.shape
        n = w.n
        if w.k != k:
            raise ValueError("x and w disagree on k")
        a = _lib.PgGemmArgs()
        a.w, a.ldw = w.data.data_ptr(), w.k
        a.x, a.ldx = x.data_ptr(), x.stride(0)
        if tp is not None:
            if mode != STORE:
                raise ValueError("a tensor-parallel GEMM publishes its tiles (store mode)")
        elif mode == RESIDUAL:
            if residual is None or residual.shape != (batch, n) or residual.stride(1) != 1:
                raise ValueError("residual mode needs residual [batch, n]")
            a.residual, a.ldr = residual.data_ptr(), residual.stride(0)
        else:
            cols = n // 2 if mode == SILU_MUL else n
            if out is None:
                out = torch.empty(batch, cols, dtype=torch.float16, device=x.device)
            if out.shape != (batch, cols) or out.stride(1) != 1:
                raise ValueError(f"out must be [batch, {cols}]")
            a.y, a.ldy = out.data_ptr(), out.stride(0)
        a.n, a.k, a.batch, a.mode, a.grid, a.pdl = n, k, batch, mode, grid, int(pdl)
        a.partials, a.partial_floats = self.partials.data_ptr(), self.partials.numel()
        a.counters, a.num_counters = self.counters.data_ptr(), self.counters.numel()
        if tp is not None:
            tp.fill(a)
        if norm_weight is not None:
            if (norm_weight.dtype != torch.float16 or norm_weight.shape != (k,)
                    or not norm_weight.is_contiguous()):
                raise ValueError(f"norm_weight must be a contiguous float16 [{k}] tensor")
            if x.data_ptr() % 16 or x.stride(0) % 8:
                raise ValueError("the normalised x must be 16-byte aligned with rows of 8k halves")
            a.norm_weight, a.norm_eps = norm_weight.data_ptr(), float(eps)
        _lib.check(_lib.load().pg_skinny_gemm(ctypes.byref(a), _stream()))
        if tp is not None:
            return None
        return out if mode != RESIDUAL else residual
