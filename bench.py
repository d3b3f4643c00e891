#!/usr/bin/env python3
"""PageGauge-B200 decode-attention benchmark (one JSON line on rank 0).

A step is one PageGauge decode attention over one layer's cache: INT8
page-affine old pages + the 256-token exact FP16 tail + LSE merge + value-
centre restore (B=1, context 49,152, Hq/Hkv 32/8,
head_dim 128, page 16).  Four layers' caches (4 x 101 MB > the 126 MB L2)
are cycled so every step streams its cache from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload b1_49k|b8_ragged|b1_4k] [--split PAGES]

With N > 1 (torchrun, one process per GPU) every rank runs its own replica
of the workload (the path has no cross-GPU exchange for one request);
``value`` is the whole-job bytes/s, timed on the device, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import threading
import time

import numpy as np
import torch

PAGE = 16
DIM = 128
HQ, HKV = 32, 8
SEED = 20261001


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("b1_49k", "b8_ragged", "b1_4k"), default="b1_49k")
    p.add_argument("--split", type=int, default=-1,
                   help="pages per work item (-1: measured scheduler table, 0: heuristic)")
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--merge", choices=("kernel", "fused"), default="kernel",
                   help="cross-CTA merge: separate merge kernel or last-CTA merge in the split kernel")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def workload_lengths(name: str, seed: int = SEED) -> list[int]:
    if name == "b1_49k":
        return [49152]
    if name == "b1_4k":
        return [4096]
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(4096, 32768 + 1, size=8)]


def algorithmic_bytes(old_tokens, exact_tokens, hkv=HKV) -> int:
    """INT8 codes (K+V) + per-(page, head) K/V scales + FP16 exact tokens."""
    total = 0
    for o, e in zip(old_tokens, exact_tokens):
        pages = o // PAGE
        total += 2 * o * hkv * DIM + pages * hkv * 2 * 2 + 2 * e * hkv * DIM * 2
    return total


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(lengths, seconds_budget: float = 15.0) -> dict:
    """The CPU oracle (float64 numpy restatement) on a bounded sample: whole
    decode steps of the same workload, request by request, until the
    budget is used (at least one request)."""
    from oracle import pagegauge_oracle as O
    from pagegauge_b200.cache import synthetic_dense_cache

    torch.set_num_threads(os.cpu_count() or 1)
    n = lengths[0]
    q, dk, dv = synthetic_dense_cache([n], seed=SEED)
    q, dk, dv = q.numpy(), dk.numpy(), dv.numpy()
    pages = n // PAGE
    tail = 16
    center_k = dk.reshape(-1, HKV, DIM).astype(np.float32).mean(0).astype(np.float16)
    center_v = dv.reshape(-1, HKV, DIM).astype(np.float32).mean(0).astype(np.float16)
    ck, sk = O.quantize_pages_bulk(dk, center_k)
    cv, sv = O.quantize_pages_bulk(dv, center_v)
    ek = (dk[pages - tail:].astype(np.float32) - center_k.astype(np.float32)).astype(np.float16)
    ev = (dv[pages - tail:].astype(np.float32) - center_v.astype(np.float32)).astype(np.float16)
    old = list(range(pages - tail))
    steps = 0
    t0 = time.perf_counter()
    while True:
        O.page_gauge_decode(q[0], ck, cv, sk, sv, old, len(old) * PAGE, ek, ev, list(range(tail)),
                            tail * PAGE, center_v, 1.0 / math.sqrt(DIM))
        steps += 1
        if time.perf_counter() - t0 > seconds_budget or steps >= 20:
            break
    dt = (time.perf_counter() - t0) / steps
    nbytes = algorithmic_bytes([len(old) * PAGE], [tail * PAGE])
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} full decode steps of B=1 ctx {n} (float64 numpy oracle), "
                      f"{dt * 1e3:.1f} ms/step"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lengths = workload_lengths(args.workload)
    if args.workload == "b8_ragged":
        lengths = lengths[:1]  # bounded: one request of the ragged batch per step
    budget = 10.0
    base = cpu_baseline(lengths, seconds_budget=budget)
    line = {
        "impl": "reference", "metric": f"decode-attn HBM GB/s ({args.workload})",
        "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp16 storage, f64 math",
        "data": "synthetic", "config": {"workload": args.workload, "lengths": lengths},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    from pagegauge_b200 import scheduler
    from pagegauge_b200.cache import build_gauge_cache, synthetic_dense_cache
    from pagegauge_b200.decode import PageGaugeDecode
    from pagegauge_b200.runtime import load_append_extension, read_device_error

    lengths = workload_lengths(args.workload)
    layers = max(1, args.layers)
    caches = []
    q = tables = None
    for layer in range(layers):
        qi, dk, dv = synthetic_dense_cache(lengths, seed=SEED + layer + 1000 * rank, device="cuda")
        cache, tables = build_gauge_cache(dk, dv, lengths)
        del dk, dv
        caches.append(cache)
        q = qi if q is None else q
    torch.cuda.synchronize()
    split = args.split
    if split < 0:
        split = scheduler.lookup(len(lengths), max(lengths))
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    dec = PageGaugeDecode(ws)
    dec.plan(tables.old_indptr, tables.old_indices, tables.exact_indptr, tables.exact_indices,
             tables.exact_last_page_len, HQ, HKV, old_split_pages=split, exact_split_pages=0)
    out = torch.empty_like(q)

    def step(layer: int):
        c = caches[layer]
        dec.run(q, c.key_codes, c.value_codes, c.key_scales, c.value_scales, c.exact_key,
                c.exact_value, c.value_center, out=out, fused_merge=args.merge == "fused")

    # Steps are captured into CUDA graphs (plan stays outside capture, as in
    # the reference): one graph of CHUNK consecutive steps cycling the
    # layers, replayed K // CHUNK times, plus single-step graphs for the
    # remainder, so host launch overhead is amortised and exactly K steps
    # are timed on the device.
    stream = torch.cuda.Stream()
    chunk = 8 * layers
    with torch.cuda.stream(stream):
        for layer in range(layers):
            step(layer)
        torch.cuda.synchronize()
        chunk_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(chunk_graph, stream=stream):
            for i in range(chunk):
                step(i % layers)
        single = []
        for layer in range(layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(layer)
            single.append(g)
    torch.cuda.synchronize()

    def run_steps(k: int) -> None:
        for _ in range(k // chunk):
            chunk_graph.replay()
        for i in range(k - k % chunk, k):
            single[i % layers].replay()

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record()
        run_steps(args.steps)
        end.record()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    nbytes = algorithmic_bytes(tables.old_tokens, tables.exact_tokens)
    value = world * nbytes / (ms * 1e-3) / 1e9
    err = read_device_error()

    # Dominant kernel alone: the split-KV decode launch (partials only), one
    # graph per layer, timed with events on the replay stream.
    plan = dec.work_plan
    lib_launches = 1 if (plan.single and plan.num_items) else 2
    from pagegauge_b200 import wrapper as W

    def decode_only(layer: int):
        c = caches[layer]
        segs = (W._segment(c.key_codes, c.value_codes, dec._old_indices, dec._old_last,
                           c.key_scales, c.value_scales),
                W._segment(c.exact_key, c.exact_value, dec._exact_indices, dec._exact_last))
        import ctypes
        from pagegauge_b200 import _lib
        a = _lib.PgDecodeArgs()
        a.q = q.data_ptr()
        a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
        a.batch, a.kv_heads, a.group = plan.batch, plan.kv_heads, plan.group
        a.sm_scale = dec.sm_scale
        a.seg[0], a.seg[1] = segs
        a.items, a.item_off, a.num_items, a.warps_per_cta = plan.items_ptr, plan.off_ptr, plan.num_items, plan.warps
        a.part_o, a.part_lse = plan.o_ptr, plan.lse_ptr
        a.final_mode = 1 if plan.single else 0
        a.out = out.data_ptr()
        a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
        a.stage_mask = 1  # split kernel only (partials; no fused merge)
        _lib.check(_lib.load().pg_decode_run(ctypes.byref(a), torch.cuda.current_stream().cuda_stream))

    with torch.cuda.stream(stream):
        kernel_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kernel_graph, stream=stream):
            for i in range(chunk):
                decode_only(i % layers)
    torch.cuda.synchronize()
    kernel_graph.replay()
    ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    kreps = max(4, args.steps // chunk)
    ks.record()
    for _ in range(kreps):
        kernel_graph.replay()
    ke.record()
    torch.cuda.synchronize()
    kernel_ms = ks.elapsed_time(ke) / (kreps * chunk)

    peaks_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        peak = json.load(open(peaks_path))["hbm_gbs"]
        peak_src = "measured"
    else:
        peak, peak_src = 6650.0, "fallback"
    achieved = nbytes / (kernel_ms * 1e-3) / 1e9
    traffic_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                                f"decode_split_kernel_{args.workload}_traffic.json")
    traffic = None
    if os.path.exists(traffic_path):
        traffic = json.load(open(traffic_path)).get("dram_bytes_per_launch")

    # End to end through the public API with host buffers: per step the new
    # token's q/k/v go host->device (pinned), the fused append writes the
    # exact ring, the decode runs, and the output comes back to the host.
    ext = load_append_extension()
    pos = lengths[0] - 1
    cos, sin = (torch.ones(DIM, dtype=torch.float16, device="cuda"),
                torch.zeros(DIM, dtype=torch.float16, device="cuda"))
    hq_in = torch.randn(len(lengths), HQ, DIM).half().pin_memory()
    hk_in = torch.randn(len(lengths), HKV, DIM).half().pin_memory()
    hv_in = torch.randn(len(lengths), HKV, DIM).half().pin_memory()
    h_out = torch.empty(len(lengths), HQ, DIM, dtype=torch.float16).pin_memory()
    dq, dk1, dv1 = torch.empty_like(q), torch.empty(len(lengths), HKV, DIM, dtype=torch.float16, device="cuda"), \
        torch.empty(len(lengths), HKV, DIM, dtype=torch.float16, device="cuda")
    rq = torch.empty_like(q)
    e2e_steps = max(10, args.steps // 4)

    def e2e_step(i):
        c = caches[i % layers]
        dq.copy_(hq_in, non_blocking=True)
        dk1.copy_(hk_in, non_blocking=True)
        dv1.copy_(hv_in, non_blocking=True)
        # The append rewrites the last token of the (exact) last page, which
        # also exercises the page-close finalisation every step.
        ext.rope_append_page_gauge(dq, dk1, dv1, cos, sin, c.key_center, c.value_center, rq,
                                   c.exact_key, c.exact_value, c.key_codes, c.value_codes,
                                   c.key_scales, c.value_scales, 0, pos)
        dec.run(rq, c.key_codes, c.value_codes, c.key_scales, c.value_scales, c.exact_key,
                c.exact_value, c.value_center, out=out)
        h_out.copy_(out, non_blocking=True)

    e2e_value = None
    if len(lengths) == 1:
        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        for i in range(e2e_steps):
            e2e_step(i)
        ee.record()
        torch.cuda.synchronize()
        e2e_ms = es.elapsed_time(ee) / e2e_steps
        e2e_value = world * nbytes / (e2e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(lengths if len(lengths) == 1 else lengths[:1])

    if rank == 0:
        line = {
            "metric": f"decode-attn HBM GB/s ({args.workload})",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "us_per_step": ms * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 codes + fp16 tail, fp16 mma / fp32 softmax",
            "data": "synthetic (seeded; K=RoPE(N(mu,1)), mu~N(0,2); V,Q~N(0,1))",
            "config": {"workload": args.workload, "lengths": lengths, "hq": HQ, "hkv": HKV,
                       "head_dim": DIM, "page": PAGE, "exact_tail_tokens": 256,
                       "split_pages": plan.split_pages[0], "work_items": plan.num_items,
                       "layers_cycled": layers,
                       "l2": f"{layers} layer caches cycled ({layers * nbytes / 1e6:.0f} MB > 126 MB L2)",
                       "parallelism": f"replicas x{world}"},
            "algorithmic_bytes_per_step": nbytes,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": peak_src, "kernel": "pg_decode_split_kernel",
                         "kernel_us": kernel_ms * 1e3},
            "gpu_launches": lib_launches * args.steps,
            "e2e": None if e2e_value is None else {
                "value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": hq_in.numel() * 2 + hk_in.numel() * 2 + hv_in.numel() * 2,
                "d2h_bytes_per_step": h_out.numel() * 2},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "device_guard": err,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        del chunk_graph, single, kernel_graph
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
