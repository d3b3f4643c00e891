"""Failure detection without a GPU fault: the peer-memory reduction waits
for every rank's tagged tiles for about a second at most, then records
PG_DEV_WAIT_TIMEOUT in the device guard word and returns, and the context
stays usable.  One GPU: this rank publishes its partial (world 2, both
buffer slots being its own buffer) and no second rank ever publishes, so
the reduce waits on tags that nothing sets, and a row that timed out
stores neither its residual nor its output."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from pagegauge_b200 import _lib
from pagegauge_b200.runtime import read_device_error

pytestmark = pytest.mark.gpu

PG_DEV_WAIT_TIMEOUT = 1
PG_TP_PAYLOAD_F16 = 1  # tiles published by pg_tp_publish


def test_tp_reduce_gives_up_when_a_rank_never_publishes(cuda_lib):
    lib = _lib.load()
    tiles, batch, n = 64, 1, 4096
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * 64)()
    _lib.check(lib.pg_tp_exchange_create(tiles, ctypes.byref(own), handle))
    try:
        assert read_device_error() == 0
        stream = torch.cuda.current_stream().cuda_stream
        src = torch.randn(batch, n, device="cuda").half()
        out = torch.full((batch, n), 7.0, device="cuda").half()
        residual = torch.randn(batch, n, device="cuda").half()
        residual_before = residual.clone()
        norm_w = torch.ones(n, device="cuda").half()
        peers = (ctypes.c_void_p * 2)(own.value, own.value)
        _lib.check(lib.pg_tp_publish(peers, 2, 0, tiles, tiles, batch, src.data_ptr(), n, stream))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _lib.check(lib.pg_tp_reduce(own, 2, tiles, tiles, batch, residual.data_ptr(), n,
                                    norm_w.data_ptr(), 1e-5, out.data_ptr(), n,
                                    PG_TP_PAYLOAD_F16, stream))
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert read_device_error() == PG_DEV_WAIT_TIMEOUT
        assert 0.5 < waited < 10.0, waited
        # The timed-out step changed nothing: the decoder can repeat it.
        assert torch.equal(residual, residual_before)
        assert bool((out == 7.0).all())
        # The context is intact: ordinary work runs and the guard is clear.
        x = torch.arange(1024, device="cuda", dtype=torch.float32)
        assert float(x.sum()) == 1023 * 1024 / 2
        assert read_device_error() == 0
    finally:
        torch.cuda.synchronize()
        _lib.check(lib.pg_tp_exchange_destroy(own))
