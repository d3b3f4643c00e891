"""Peer-memory exchange buffers for the tensor-parallel projections.

The decoder's row-parallel projections (o_proj and down_proj under tensor
parallelism, scripts/benchmark_page_gauge_transformer.py:2754-2804) end in
an all-reduce of a [B, hidden] partial product.  Here no collective library
is involved: the projection GEMM publishes every finished FP32 output tile
into every rank's exchange buffer as soon as the tile is done (plain peer
stores over NVLink, every value tagged with the exchange count, so the
transfer overlaps the rest of the GEMM), or ``publish`` does the same for a
partial another GEMM (cuBLAS) wrote, as FP16 pairs (half the bytes, since
every rank sends its whole partial to every other rank); the next kernel
on each rank waits
(bounded) for all ranks' tiles, sums them in rank order and applies the
residual add and RMSNorm (``reduce``).  This module allocates one
exchange buffer per rank (CUDA IPC), shares the handles over the process
group and maps the other ranks' buffers.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

# pg_tp_reduce's payload argument (PG_TP_PAYLOAD_* in the C header).
PAYLOAD_F32 = 0  # tiles published by a tensor-parallel streaming GEMM
PAYLOAD_F16 = 1  # tiles published by pg_tp_publish


class TpExchange:
    """One rank's exchange buffer plus every other rank's, mapped here.

    ``tiles_cap`` = output tiles of 64 rows the largest exchanged GEMM has
    (hidden / 64).  Every rank must construct it (collective), and ``close``
    it (collective) before the process group is destroyed."""

    MAX_RANKS = 8

    def __init__(self, process_group, tiles_cap: int, device: torch.device | str = "cuda"):
        import torch.distributed as dist

        self.group = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if not 2 <= self.world <= self.MAX_RANKS:
            raise ValueError(f"peer-memory reduction supports 2..{self.MAX_RANKS} ranks")
        self.tiles_cap = int(tiles_cap)
        lib = _lib.load()
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(torch.device(device)):
            _lib.check(lib.pg_tp_exchange_create(self.tiles_cap, ctypes.byref(own), handle))
        self.own = int(own.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=process_group)
        self.peers: list[int] = []
        self._opened: list[int] = []
        try:
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peers.append(self.own)
                    continue
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                ptr = ctypes.c_void_p()
                _lib.check(lib.pg_tp_exchange_open(buf, ctypes.byref(ptr)))
                self.peers.append(int(ptr.value))
                self._opened.append(int(ptr.value))
        except Exception:
            self._release()
            raise
        dist.barrier(group=process_group)
        self.closed = False
        # Format of the tiles the next reduce sums: FP32 pairs from a
        # publishing streaming GEMM (``fill``), FP16 pairs from ``publish``.
        self.payload = PAYLOAD_F32

    def fill(self, args) -> None:
        """Set the tensor-parallel fields of a PgGemmArgs."""
        args.tp_world, args.tp_rank, args.tp_tiles_cap = self.world, self.rank, self.tiles_cap
        for r, ptr in enumerate(self.peers):
            args.tp_peers[r] = ptr
        self.payload = PAYLOAD_F32

    def publish(self, src: torch.Tensor) -> None:
        """Publish this rank's partial product computed by another GEMM
        (float16 [batch, tiles * 64], e.g. cuBLAS's row-parallel output) to
        every rank, as a tensor-parallel streaming GEMM publishes its tiles;
        the next ``reduce`` sums the ranks' partials."""
        if src.dtype != torch.float16 or src.dim() != 2 or src.stride(1) != 1:
            raise ValueError("src must be a float16 [batch, n] tensor with contiguous rows")
        if src.shape[1] % 64 or src.shape[1] // 64 > self.tiles_cap:
            raise ValueError(f"src columns must be a multiple of 64, at most {self.tiles_cap * 64}")
        peers = (ctypes.c_void_p * self.world)(*self.peers)
        _lib.check(_lib.load().pg_tp_publish(
            peers, self.world, self.rank, self.tiles_cap, src.shape[1] // 64, src.shape[0],
            src.data_ptr(), src.stride(0), torch.cuda.current_stream(src.device).cuda_stream))
        self.payload = PAYLOAD_F16

    def reduce(self, batch: int, residual: torch.Tensor | None, norm_weight: torch.Tensor | None,
               eps: float, out: torch.Tensor, tiles: int | None = None) -> torch.Tensor:
        """Sum the ranks' published tiles of the last tensor-parallel GEMM on
        this rank (waits for them, bounded); with ``residual``: residual +=
        f16(sum), out = RMSNorm(residual) (``norm_weight``) or the residual;
        without: out = f16(sum).  ``tiles`` = output columns / 64 of that
        GEMM (default: the capacity)."""
        tiles = self.tiles_cap if tiles is None else int(tiles)
        if out.dtype != torch.float16 or out.dim() != 2 or out.stride(1) != 1:
            raise ValueError("out must be a float16 [batch, n] tensor with contiguous rows")
        if out.shape != (batch, tiles * 64):
            raise ValueError(f"out must be [{batch}, {tiles * 64}]")
        if residual is not None and (residual.shape != out.shape or residual.stride(1) != 1
                                     or residual.dtype != torch.float16):
            raise ValueError("residual must match out")
        _lib.check(_lib.load().pg_tp_reduce(
            ctypes.c_void_p(self.own), self.world, self.tiles_cap, tiles, batch,
            None if residual is None else residual.data_ptr(),
            0 if residual is None else residual.stride(0),
            None if norm_weight is None else norm_weight.data_ptr(), float(eps),
            out.data_ptr(), out.stride(0), self.payload,
            torch.cuda.current_stream(out.device).cuda_stream))
        return out

    def _release(self) -> None:
        lib = _lib.load()
        for ptr in self._opened:
            lib.pg_tp_exchange_close(ctypes.c_void_p(ptr))
        self._opened = []
        if self.own:
            lib.pg_tp_exchange_destroy(ctypes.c_void_p(self.own))
            self.own = 0

    def close(self) -> None:
        """Collective: unmap the other ranks' buffers, then free this rank's
        once no rank can still write into it."""
        import torch.distributed as dist

        if self.closed:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = _lib.load()
        for ptr in self._opened:
            _lib.check(lib.pg_tp_exchange_close(ctypes.c_void_p(ptr)))
        self._opened = []
        dist.barrier(group=self.group)
        _lib.check(lib.pg_tp_exchange_destroy(ctypes.c_void_p(self.own)))
        self.own = 0
        self.closed = True
