"""The streaming GEMM's peer-memory tensor-parallel reduction on 2, 4 and 8 GPUs:
each rank multiplies its K-slice and publishes every finished tile into
the ranks' exchange buffers (NVLink peer stores + arrival flags); the
reduce kernel waits (bounded) for all ranks' tiles, sums them in rank order
and applies the residual add / RMSNorm.  Every rank must end with the
same bits, within the FP32-accumulation tolerance of the full product, over
consecutive launches (both halves of the double-buffered exchange) and CUDA
graph replays; a partial another GEMM computed (FP16) goes through
pg_tp_publish and must reduce to the FP32 rank-order sum bit for bit.
The reduce kernel reads the ranks' tiles four ranks per
memory round trip, so 8 ranks take two batches and 2 one partial batch.
Each rank count is skipped unless that many GPUs are visible."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, result, batch, n, k):
    import torch.distributed as dist

    from pagegauge_b200.gemm import STORE, PackedWeight, SkinnyGemm
    from pagegauge_b200.peer import TpExchange
    from pagegauge_b200.runtime import read_device_error

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(5)
        w = (torch.randn(n, k, generator=g) * 0.02).half()
        x = torch.randn(batch, k, generator=g).half()
        r0 = torch.randn(batch, n, generator=g).half()
        ks = k // world
        wl = w[:, rank * ks:(rank + 1) * ks].contiguous().cuda()
        xl = x[:, rank * ks:(rank + 1) * ks].contiguous().cuda()
        tpx = TpExchange(dist.group.WORLD, n // 64, "cuda")
        gemm = SkinnyGemm("cuda")
        gemm.reserve(n, ks, batch, STORE)
        pw = PackedWeight(wl)
        tiles = n // 64

        def run(out, residual=None, norm=None):
            gemm(xl, pw, tp=tpx)  # publishes this rank's tiles
            tpx.reduce(batch, residual, norm, 1e-5, out, tiles)

        outs = []
        for _ in range(3):  # consecutive launches alternate exchange halves
            y = torch.empty(batch, n, dtype=torch.float16, device="cuda")
            run(y)
            outs.append(y)
        res = r0.cuda()
        run(res, residual=res)
        nw = (1 + 0.1 * torch.randn(n, generator=g)).half().cuda()
        res2 = r0.cuda()
        normed = torch.empty(batch, n, dtype=torch.float16, device="cuda")
        run(normed, residual=res2, norm=nw)
        s = torch.cuda.Stream()
        y = torch.empty(batch, n, dtype=torch.float16, device="cuda")
        with torch.cuda.stream(s):
            run(y)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                run(y)
            for _ in range(5):
                y.zero_()
                graph.replay()
        torch.cuda.synchronize()
        del graph
        # A partial computed by another GEMM (torch / cuBLAS, FP16) goes
        # through pg_tp_publish (FP16-pair payload), twice in a row so both
        # halves of the exchange carry it.
        part = (xl.float() @ wl.float().t()).half()
        pubs = []
        for _ in range(2):
            z = torch.empty(batch, n, dtype=torch.float16, device="cuda")
            tpx.publish(part)
            tpx.reduce(batch, None, None, 1e-5, z, tiles)
            pubs.append(z)
        torch.cuda.synchronize()
        err = read_device_error()
        gathered = [None] * world
        dist.all_gather_object(gathered, {"outs": [o.cpu().numpy() for o in outs],
                                          "res": res.cpu().numpy(), "graph": y.cpu().numpy(),
                                          "res2": res2.cpu().numpy(),
                                          "normed": normed.cpu().numpy(), "err": err,
                                          "part": part.cpu().numpy(),
                                          "pub": np.stack([z.cpu().numpy() for z in pubs])})
        if rank == 0:
            np.savez(result, w=w.numpy(), x=x.numpy(), r0=r0.numpy(), nw=nw.cpu().numpy(),
                     **{f"r{i}_{k_}": v for i, d in enumerate(gathered)
                        for k_, v in (("outs", np.stack(d["outs"])), ("res", d["res"]),
                                      ("graph", d["graph"]), ("res2", d["res2"]),
                                      ("normed", d["normed"]), ("err", np.array(d["err"])),
                                      ("part", d["part"]), ("pub", d["pub"]))})
        tpx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("batch,n,k", [(1, 4096, 4096), (5, 1024, 2048), (16, 512, 1024)])
def test_peer_memory_reduction(cuda_lib, tmp_path, world, batch, n, k):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        port = sck.getsockname()[1]
    path = str(tmp_path / "tp.npz")
    mp.spawn(_rank, args=(world, port, path, batch, n, k), nprocs=world, join=True)
    d = np.load(path)
    assert all(int(d[f"r{r}_err"]) == 0 for r in range(world))
    # Published FP16 partials: the FP32 sum in rank order, rounded to FP16,
    # bit for bit on every rank and in both halves of the exchange.
    acc = np.zeros_like(d["r0_part"], dtype=np.float32)
    for r in range(world):
        acc += d[f"r{r}_part"].astype(np.float32)
    for r in range(world):
        for z in d[f"r{r}_pub"]:
            assert np.array_equal(z, acc.astype(np.float16))
    ref = d["x"].astype(np.float64) @ d["w"].astype(np.float64).T
    for r in range(world):
        outs = d[f"r{r}_outs"]
        assert all(np.array_equal(outs[0], o) for o in outs[1:])
        assert np.array_equal(outs[0], d["r0_outs"][0])  # identical on every rank
        assert np.array_equal(d[f"r{r}_graph"], outs[0])
        tol = np.abs(ref) * 2.0 ** -10 + 1e-6 * np.sqrt(k)
        assert np.all(np.abs(outs[0].astype(np.float64) - ref) <= tol)
        res = (d["r0"].astype(np.float32) + outs[0].astype(np.float32)).astype(np.float16)
        assert np.array_equal(d[f"r{r}_res"], res)
        assert np.array_equal(d[f"r{r}_res2"], res)
        # RMSNorm of the updated residual (MistralRMSNorm rounding points).
        xf = res.astype(np.float32)
        inv = 1 / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-5)
        exp = (d["nw"].astype(np.float32) * (xf * inv).astype(np.float16).astype(np.float32))
        got = d[f"r{r}_normed"].astype(np.float32)
        assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -9 + 1e-6)
        assert np.array_equal(d[f"r{r}_normed"], d["r0_normed"])
