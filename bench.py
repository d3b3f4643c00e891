#!/usr/bin/env python3
"""PageGauge-B200 decode benchmark (one JSON line on rank 0).

A step is one PageGauge decode attention over one layer's cache: INT8
page-affine old pages + the 256-token exact FP16 tail + LSE merge + value-
centre restore, 32 Q / 8 KV heads, head_dim 128, page 16.  The headline
workload is B1/49K (B=1, context 49,152); several layers' caches (more
bytes than the 126 MB L2, values drawn from the three benchmark seeds) are
cycled so every step streams its cache from HBM.  The same line carries,
under ``workloads``, measured in the same run (``--only`` skips them):

* ``b8_ragged``: the 8 ragged requests (lengths and values from each of
  the three seeds), sharded over the ranks (strong scaling);
* ``append_b8_32l``: the fused append step (B=8, 32 layers);
* ``affine_group16_*``: the alternative page representation;
* ``decoder_b1`` / ``decoder_b32``: the Mistral-7B-shaped decoder's
  tokens/s at context 16K, tensor-parallel over the ranks (strong).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload b1_49k|b8_ragged|b1_4k|decoder|gemm] [--split PAGES] [--only]

``e2e`` is the same step through the public API with host buffers: the
append reads each step's q/k/v from page-locked host memory and the decode
writes the output there, every step, in CUDA graphs of 32 steps (plus the
remainder), exactly K steps timed.

Multi-GPU (torchrun, one process per GPU): B1/49K and B1/4K run one replica
per rank (weak scaling, no data-path collective); B8 ragged splits its 8
requests over the ranks by request (longest-first bin packing on decode
bytes) or by KV head, whichever balances the bytes (strong scaling, no
data-path collective); the decoder is tensor-parallel by KV head.
``value`` is the whole-job bytes/s: all ranks' bytes over the max-over-ranks
device time.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

PAGE = 16
DIM = 128
HQ, HKV = 32, 8
SEED = 20261001
SEEDS = (20261001, 20261002, 20261003)  # the benchmark configs' three seeds
TAIL_PAGES = 16
L2_BYTES = 126 << 20


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload",
                   choices=("b1_49k", "b8_ragged", "b1_4k", "decoder", "gemm", "append"),
                   default="b1_49k")
    p.add_argument("--split", type=int, default=-1,
                   help="pages per work item (-1: measured scheduler table, 0: heuristic)")
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--warps", type=int, default=4, help="warps per split-KV CTA")
    p.add_argument("--merge", choices=("kernel", "fused", "cluster"), default="kernel",
                   help="cross-CTA merge: separate merge kernel, last-CTA merge, or a single "
                        "launch merging in thread-block clusters")
    p.add_argument("--cluster", type=int, default=4, help="cluster size for --merge cluster")
    p.add_argument("--only", action="store_true", help="skip the secondary workloads")
    p.add_argument("--decoder-batch", type=int, nargs="*", default=[32, 1],
                   help="decoder workload: batch sizes (the first is the headline)")
    p.add_argument("--decoder-steps", type=int, default=16)
    p.add_argument("--decoder-policy", default="S0/A0/T256",
                   help="exact pages: S<sink pages>/A<static suffix pages>/T<tail tokens>")
    p.add_argument("--decoder-tp-reduce", choices=("peer", "nccl"), default="peer",
                   help="tensor-parallel reduction of the streaming projections")
    p.add_argument("--decoder-gemm", choices=("auto", "pg", "cublas"), default="auto",
                   help="decoder projections: weight-streaming kernels (pg), cuBLAS, or by batch")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


# ----------------------------------------------------------------- helpers
def algorithmic_bytes(old_tokens, exact_tokens, hkv=HKV) -> int:
    """INT8 codes (K+V) + per-(page, head) K/V scales + FP16 exact tokens."""
    total = 0
    for o, e in zip(old_tokens, exact_tokens):
        pages = o // PAGE
        total += 2 * o * hkv * DIM + pages * hkv * 2 * 2 + 2 * e * hkv * DIM * 2
    return total


def global_lengths(name: str, seed: int = SEED) -> list[int]:
    """Request lengths of a workload (all ranks together)."""
    from pagegauge_b200.shard import ragged_lengths

    if name == "b1_49k":
        return [49152]
    if name == "b1_4k":
        return [4096]
    return ragged_lengths(8, seed)


def workload_bytes(lengths) -> int:
    """Algorithmic bytes of one decode step over ``lengths`` (the last
    TAIL_PAGES pages of each request exact FP16, the rest INT8)."""
    old, exact = [], []
    for n in lengths:
        pages = -(-n // PAGE)
        n_old = max(pages - TAIL_PAGES, 0)
        old.append(n_old * PAGE)
        exact.append(n - n_old * PAGE)
    return algorithmic_bytes(old, exact)


def workload_lengths(name: str, world: int = 1, rank: int = 0, seed: int = SEED):
    """(this rank's request lengths, global lengths, shards or None).
    B1 workloads are replicas (every rank runs the whole request); B8
    ragged shards its 8 requests over the ranks."""
    from pagegauge_b200.shard import shard_requests

    glob = global_lengths(name, seed)
    if name in ("b1_49k", "b1_4k"):
        return list(glob), glob, None
    shards = shard_requests(glob, world)
    return [glob[i] for i in shards[rank]], glob, shards


def workload_config(args, world: int) -> dict:
    """The ``config`` both arms print, identical for the same command line:
    the workload's shape, seeds, how the L2 is kept out of the timing, and
    how it is split over GPUs."""
    lengths = global_lengths(args.workload)
    nbytes = workload_bytes(lengths)
    replicas = args.workload in ("b1_49k", "b1_4k")
    return {
        "workload": args.workload, "lengths": lengths, "hq": HQ, "hkv": HKV, "head_dim": DIM,
        "page": PAGE, "exact_tail_tokens": TAIL_PAGES * PAGE, "seeds": list(SEEDS),
        "l2": (f"{args.layers} layer caches cycled (values from the seeds in turn), "
               f"{args.layers * nbytes / 1e6:.0f} MB > 126 MB L2: each step reads its cache "
               f"from HBM"),
        "parallelism": (f"replicas x{world} (weak)" if replicas
                        else f"requests sharded over {world} GPU(s) (strong)"),
    }


def upload_graph(graph) -> None:
    """Upload a captured CUDA graph to the device (cuGraphUpload) so that its
    first replay -- which may be the timed one -- launches like any later
    replay instead of paying the one-time upload."""
    handle = graph.raw_cuda_graph_exec()
    stream = torch.cuda.current_stream().cuda_stream
    rc = ctypes.CDLL("libcuda.so.1").cuGraphUpload(ctypes.c_void_p(int(handle)),
                                                    ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"cuGraphUpload failed ({rc})")
    torch.cuda.synchronize()


class Dist:
    """Barrier / max / sum over ranks (no-ops for one process)."""

    def __init__(self, world: int):
        self.world = world
        if world > 1:
            import torch.distributed as dist
            self.dist = dist
        else:
            self.dist = None

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def reduce(self, x: float, op: str) -> float:
        if self.dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX if op == "max" else self.dist.ReduceOp.SUM)
        return float(t.item())


def peak_hbm():
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    if os.path.exists(path):
        return float(json.load(open(path))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(workload: str):
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                        f"decode_split_kernel_{workload}_traffic.json")
    if os.path.exists(path):
        return json.load(open(path)).get("dram_bytes_per_launch")
    return None


class ClockSampler:
    """nvidia-smi sampling (every 100 ms) across the whole measured phase:
    the headline steps, the kernel-only graphs, the end-to-end runs and the
    secondary workloads (a single timed region is far shorter than one
    sampling period)."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        return self.__enter__()

    def stop(self):
        self.__exit__(None, None, None)

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


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(lengths, seconds_budget: float = 15.0) -> dict:
    """The CPU oracle (float64 numpy restatement) on a bounded sample: whole
    decode steps of the first request of the workload until the budget is
    used (at least one step)."""
    torch.set_num_threads(os.cpu_count() or 1)
    fn, nbytes = reference_decode_sample(lengths[:1], SEED)
    steps = 0
    t0 = time.perf_counter()
    while True:
        fn()
        steps += 1
        if time.perf_counter() - t0 > seconds_budget or steps >= 20:
            break
    dt = (time.perf_counter() - t0) / steps
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{steps} full decode steps of one request, ctx {lengths[0]} (float64 numpy "
                      f"oracle, {torch.get_num_threads()} threads), {dt * 1e3:.1f} ms/step",
            "ms_per_step": dt * 1e3}


def decoder_cpu_baseline(context: int = 16384, seed: int = 20261004) -> dict:
    """The decoder oracle on the host cores, bounded sample: one decode step
    (B=1, position ``context``) of a one-layer model of the benchmark
    decoder's shape on a PageGauge cache of ``context`` tokens, plus the LM head alone;
    a 32-layer step is 32 layers + one head."""
    from oracle import decoder_oracle as D
    from oracle import pagegauge_oracle as O
    from pagegauge_b200.cache import rope_tables, synthetic_dense_cache
    from pagegauge_b200.decoder import (DecoderConfig, TensorParallel, full_layer_tensors,
                                        full_model_tensors, shard_layer)

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = DecoderConfig.mistral_7b_shaped()
    tp = TensorParallel.of(cfg)
    lw = shard_layer(cfg, tp, full_layer_tensors(cfg, seed, 0, "cpu"))
    top = full_model_tensors(cfg, seed, "cpu")
    w = {"embed": top["embed"].numpy(), "final_norm": top["final_norm"].numpy(),
         "lm_head": top["lm_head"].numpy(),
         "layers": [{k: getattr(lw, k).numpy() for k in
                     ("attn_norm", "qkv", "o", "mlp_norm", "gate_up", "down")}]}
    _, dk, dv = synthetic_dense_cache([context], seed=SEED)
    dk, dv = dk.numpy(), dv.numpy()
    pages = context // PAGE
    cap = pages + 1
    ck = dk.reshape(-1, HKV, DIM).astype(np.float32).mean(0).astype(np.float16)
    cv = dv.reshape(-1, HKV, DIM).astype(np.float32).mean(0).astype(np.float16)
    codes_k = np.zeros((cap, PAGE, HKV, DIM), np.int8)
    codes_v = np.zeros_like(codes_k)
    sk = np.zeros((cap, HKV), np.float16)
    sv = np.zeros_like(sk)
    codes_k[:pages], sk[:pages] = O.quantize_pages_bulk(dk, ck)
    codes_v[:pages], sv[:pages] = O.quantize_pages_bulk(dv, cv)
    ring_k = np.zeros((TAIL_PAGES, PAGE, HKV, DIM), np.float16)
    ring_v = np.zeros_like(ring_k)
    for lp in range(pages - TAIL_PAGES, pages):
        ring_k[lp % TAIL_PAGES] = (dk[lp].astype(np.float32) - ck.astype(np.float32)).astype(np.float16)
        ring_v[lp % TAIL_PAGES] = (dv[lp].astype(np.float32) - cv.astype(np.float32)).astype(np.float16)
    caches = [{"state": O.GaugeState(ring_k, ring_v, codes_k, codes_v, sk, sv),
               "key_center": ck[None], "value_center": cv[None]}]
    cos, sin = rope_tables(cap * PAGE)
    ocfg = {"hq": HQ, "hkv": HKV, "eps": cfg.rms_eps, "rope": (cos.numpy(), sin.numpy())}
    t0 = time.perf_counter()
    D.decode_step(w, ocfg, caches, [7], [context], cap)
    t_one = time.perf_counter() - t0
    x = np.ones((1, cfg.hidden), np.float16)
    t0 = time.perf_counter()
    D.linear(D.rms_norm(x, w["final_norm"], cfg.rms_eps), w["lm_head"])
    t_head = time.perf_counter() - t0
    t_step = cfg.layers * max(t_one - t_head, 0.0) + t_head
    return {"value": 1.0 / t_step, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"one decode step of a 1-layer Mistral-7B-shaped model at ctx {context} "
                      f"(numpy oracle, {torch.get_num_threads()} threads): {t_one:.2f} s, LM head "
                      f"{t_head:.2f} s; 32-layer step = 32 layers + head = {t_step:.1f} s"}


def reference_decode_sample(lengths, seed: int):
    """One request's PageGauge cache as the CPU oracle reads it (float64
    numpy restatement of the reference path): returns a function running
    one whole decode step of that request, and its algorithmic bytes."""
    from oracle import pagegauge_oracle as O
    from pagegauge_b200.cache import synthetic_dense_cache

    n = lengths[0]
    q, dk, dv = synthetic_dense_cache([n], seed=seed)
    q, dk, dv = q.numpy(), dk.numpy(), dv.numpy()
    pages = -(-n // PAGE)
    tail = min(TAIL_PAGES, pages)
    center_k = dk.reshape(-1, HKV, DIM)[:n].astype(np.float32).mean(0).astype(np.float16)
    center_v = dv.reshape(-1, HKV, DIM)[:n].astype(np.float32).mean(0).astype(np.float16)
    ck, sk = O.quantize_pages_bulk(dk, center_k)
    cv, sv = O.quantize_pages_bulk(dv, center_v)
    ek = (dk[pages - tail:].astype(np.float32) - center_k.astype(np.float32)).astype(np.float16)
    ev = (dv[pages - tail:].astype(np.float32) - center_v.astype(np.float32)).astype(np.float16)
    old = list(range(pages - tail))
    exact_tokens = n - len(old) * PAGE

    def step():
        O.page_gauge_decode(q[0], ck, cv, sk, sv, old, len(old) * PAGE, ek, ev,
                            list(range(tail)), exact_tokens, center_v, 1.0 / math.sqrt(DIM))

    return step, algorithmic_bytes([len(old) * PAGE], [exact_tokens])


def run_reference(args) -> None:
    """The reference arm: the reference's path restated on the CPU (the
    oracle port: float64 numpy, all host threads) on this box's host cores,
    rank 0 only; ``--warmup`` untimed then exactly ``--steps`` timed steps,
    each step one whole decode of a request of the workload (B1 workloads:
    the request; B8 ragged: the requests in turn), same config as the GPU
    arm."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    if args.workload == "decoder":
        base = decoder_cpu_baseline()
        print(json.dumps({
            "impl": "reference", "metric": "decoder tokens/s (Mistral-7B-shaped, B=32, ctx 16384)",
            "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": 1,
            "warmup": 0, "ms_per_step": 1e3 / base["value"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 storage, f32/f64 math",
            "data": "synthetic", "config": {"workload": "decoder", "batch": 1, "context": 16384},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    glob = global_lengths(args.workload)
    samples = [reference_decode_sample([glob[i]], SEEDS[i % len(SEEDS)])
               for i in range(len(glob))]
    for i in range(args.warmup):
        samples[i % len(samples)][0]()
    total_bytes, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        fn, nbytes = samples[i % len(samples)]
        fn()
        total_bytes += nbytes
    dt = time.perf_counter() - t0
    value = total_bytes / dt / 1e9
    sample = (f"{args.steps} timed decode steps after {args.warmup} warm-up steps, each one whole "
              f"request of the workload ({'the request' if len(glob) == 1 else 'the 8 requests in turn'}; "
              f"float64 numpy oracle, {torch.get_num_threads()} threads), "
              f"{dt / args.steps * 1e3:.1f} ms/step")
    line = {
        "impl": "reference", "metric": f"decode-attn HBM GB/s ({args.workload})",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak" if args.workload in ("b1_49k", "b1_4k") else "strong",
        "vs_baseline": None, "dtype": "int8/fp16 storage, f64 math",
        "data": "synthetic (seeded; K=RoPE(N(mu,1)), mu~N(0,2); V,Q~N(0,1))",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------- attention bench
class AttentionBench:
    """One workload's caches (``layers`` copies), its plan, and CUDA graphs
    of the public-API decode step."""

    def __init__(self, lengths, layers: int, split: int, fused_merge: bool, seed: int,
                 warps: int = 4, cluster: int = 0, hkv: int = HKV):
        from pagegauge_b200 import scheduler
        from pagegauge_b200.cache import build_gauge_cache, rope_tables, synthetic_dense_cache
        from pagegauge_b200.decode import PageGaugeDecode

        self.lengths = lengths
        self.layers = max(1, layers)
        self.fused = fused_merge
        self.cluster = cluster
        cap = max(-(-n // PAGE) for n in lengths)
        self.caches = []
        self.q = self.tables = None
        for layer in range(self.layers):
            # layer copies take their values from the benchmark seeds in turn
            qi, dk, dv = synthetic_dense_cache(lengths, hkv=hkv, seed=seed + layer % len(SEEDS),
                                               device="cuda")
            cache, tables = build_gauge_cache(dk, dv, lengths, capacity_pages=cap)
            del dk, dv
            self.caches.append(cache)
            self.q = qi if self.q is None else self.q
            self.tables = tables
        self.capacity_pages = cap
        torch.cuda.synchronize()
        if split < 0:
            split = scheduler.lookup(len(lengths), max(lengths), kv_heads=hkv)
        self.ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.dec = PageGaugeDecode(self.ws, warps_per_cta=warps)
        t = self.tables
        self.dec.plan(t.old_indptr, t.old_indices, t.exact_indptr, t.exact_indices,
                      t.exact_last_page_len, 4 * hkv, hkv, old_split_pages=split,
                      exact_split_pages=0)
        self.plan = self.dec.work_plan
        self.out = torch.empty_like(self.q)
        self.nbytes = algorithmic_bytes(t.old_tokens, t.exact_tokens, hkv=hkv)
        self.launches_per_step = 1 if ((self.plan.single and self.plan.num_items)
                                       or fused_merge or cluster > 1) else 2
        self.rope = rope_tables(cap * PAGE, device="cuda")
        self.stream = torch.cuda.Stream()
        self.chunk = 8 * self.layers

    def step(self, layer: int, q=None, out=None):
        c = self.caches[layer]
        self.dec.run(self.q if q is None else q, c.key_codes, c.value_codes, c.key_scales,
                     c.value_scales, c.exact_key, c.exact_value, c.value_center,
                     out=self.out if out is None else out, fused_merge=self.fused,
                     cluster=self.cluster)

    def capture(self):
        with torch.cuda.stream(self.stream):
            for layer in range(self.layers):
                self.step(layer)
            torch.cuda.synchronize()
            self.chunk_graph = self._graph(self.chunk)
        self.rest = {}
        torch.cuda.synchronize()

    def _graph(self, n: int):
        """A CUDA graph of n back-to-back steps cycling the layers from 0,
        uploaded to the device."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            for i in range(n):
                self.step(i % self.layers)
        upload_graph(g)
        return g

    def prepare_steps(self, k: int) -> None:
        """Capture the graph of the k % chunk remainder (outside timing)."""
        r = k % self.chunk
        if r and r not in self.rest:
            with torch.cuda.stream(self.stream):
                self.rest[r] = self._graph(r)
            torch.cuda.synchronize()

    def run_steps(self, k: int) -> None:
        """Exactly k steps cycling the layers: graphs of ``chunk`` steps
        (a multiple of the layer count), then one graph of the remainder,
        so even k < chunk runs as one graph of back-to-back steps."""
        for _ in range(k // self.chunk):
            self.chunk_graph.replay()
        if k % self.chunk:
            self.rest[k % self.chunk].replay()

    def time_steps(self, steps: int, warmup: int, dist: Dist, clocks=None) -> float:
        self.prepare_steps(max(warmup, 3))
        self.prepare_steps(steps)
        self.run_steps(max(warmup, 3))
        torch.cuda.synchronize()
        dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx = clocks if clocks is not None else _Null()
        with ctx:
            torch.cuda.synchronize()
            start.record()
            self.run_steps(steps)
            end.record()
            torch.cuda.synchronize()
        dist.barrier()
        return dist.reduce(start.elapsed_time(end) / steps, "max")

    def layer_tensors(self, layer: int):
        """(key codes, value codes, key scales, value scales, exact key,
        exact value, (k_bias, v_bias) or None) of one layer copy."""
        c = self.caches[layer]
        return (c.key_codes, c.value_codes, c.key_scales, c.value_scales, c.exact_key,
                c.exact_value, None)

    def kernel_ms(self, steps: int) -> float:
        """The split-KV decode kernel alone (partials only), graphs of
        ``chunk`` launches cycling the layers, CUDA events on the replay
        stream."""
        from pagegauge_b200 import _lib
        from pagegauge_b200 import wrapper as W

        plan, dec, q, out = self.plan, self.dec, self.q, self.out
        lib = _lib.load()
        blocks = []
        for layer in range(self.layers):
            kc, vc, ks, vs, ek, ev, affine = self.layer_tensors(layer)
            a = _lib.PgDecodeArgs()
            a.q = q.data_ptr()
            a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
            a.batch, a.kv_heads, a.group = plan.batch, plan.kv_heads, plan.group
            a.sm_scale = dec.sm_scale
            a.seg[0] = W._segment(kc, vc, dec._old_indices, dec._old_last, ks, vs)
            a.seg[1] = W._segment(ek, ev, dec._exact_indices, dec._exact_last)
            if affine is not None:
                a.representation = 1
                a.k_bias, a.v_bias = affine[0].data_ptr(), affine[1].data_ptr()
            a.items, a.item_off, a.num_items = plan.items_ptr, plan.off_ptr, plan.num_items
            a.warps_per_cta = plan.warps
            a.part_o, a.part_lse = plan.o_ptr, plan.lse_ptr
            a.final_mode = 1 if plan.single else 0
            a.out = out.data_ptr()
            a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
            a.stage_mask = 1  # split kernel only
            blocks.append(a)
        with torch.cuda.stream(self.stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                for i in range(self.chunk):
                    _lib.check(lib.pg_decode_run(ctypes.byref(blocks[i % self.layers]),
                                                 torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        g.replay()
        reps = max(4, steps // self.chunk)
        ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ks.record()
        for _ in range(reps):
            g.replay()
        ke.record()
        torch.cuda.synchronize()
        del g
        return ks.elapsed_time(ke) / (reps * self.chunk)

    def e2e(self, steps: int, dist: Dist) -> dict:
        """End to end through the public API with host buffers: per step
        the new token's q/k/v of every request go host->device from pinned
        memory, the fused RoPE/append (per-request positions) writes the
        exact ring and closes the page of requests at a page end, the
        decode runs, and the output comes back to pinned host memory.
        Reported for a CUDA graph of that public-API sequence (how the
        reference drives its decode step) and for eager calls."""
        from pagegauge_b200.runtime import load_append_extension

        ext = load_append_extension()
        B = len(self.lengths)
        g = torch.Generator().manual_seed(SEED + 77)
        # The new token's q | k | v rows packed per request (the layout of a
        # fused qkv projection), one host->device copy per step.
        width = (HQ + 2 * HKV) * DIM
        hqkv = torch.randn(B, width, generator=g).half().pin_memory()
        hout = torch.empty(B, HQ, DIM, dtype=torch.float16).pin_memory()
        dqkv = torch.empty(B, width, dtype=torch.float16, device="cuda")
        dq = dqkv[:, :HQ * DIM].view(B, HQ, DIM)
        dk = dqkv[:, HQ * DIM:(HQ + HKV) * DIM].view(B, HKV, DIM)
        dv = dqkv[:, (HQ + HKV) * DIM:].view(B, HKV, DIM)
        rq = torch.empty(B, HQ, DIM, dtype=torch.float16, device="cuda")
        out = torch.empty_like(rq)
        # Each step re-appends the last token of every request (its page
        # stays in the exact window), so the cache shape is unchanged.
        positions = torch.tensor([n - 1 for n in self.lengths], dtype=torch.int32, device="cuda")
        cos, sin = self.rope

        def one(layer: int):
            c = self.caches[layer]
            dqkv.copy_(hqkv, non_blocking=True)
            ext.rope_append_page_gauge_batched(dq, dk, dv, cos, sin, positions, c.key_center,
                                               c.value_center, rq, c.exact_key, c.exact_value,
                                               c.key_codes, c.value_codes, c.key_scales,
                                               c.value_scales, 0)
            self.step(layer, q=rq, out=out)
            hout.copy_(out, non_blocking=True)

        # Zero copy: the append reads the pinned host q|k|v rows and the
        # merge writes the output into pinned host memory, both over the
        # host link inside the kernels (no copy launches in the step).
        hq = hqkv[:, :HQ * DIM].view(B, HQ, DIM)
        hk = hqkv[:, HQ * DIM:(HQ + HKV) * DIM].view(B, HKV, DIM)
        hv = hqkv[:, (HQ + HKV) * DIM:].view(B, HKV, DIM)

        def one_zero_copy(layer: int):
            # The host rows are written before the graph and by no kernel:
            # the append may request them before waiting for the previous
            # step's kernels (each step still reads them over the host link).
            c = self.caches[layer]
            ext.rope_append_page_gauge_batched(hq, hk, hv, cos, sin, positions, c.key_center,
                                               c.value_center, rq, c.exact_key, c.exact_value,
                                               c.key_codes, c.value_codes, c.key_scales,
                                               c.value_scales, 0, inputs_ready=True)
            self.step(layer, q=rq, out=hout)

        def timed(fn, n):
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            dist.barrier()
            es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            es.record()
            for i in range(n):
                fn(i)
            ee.record()
            torch.cuda.synchronize()
            dist.barrier()
            return dist.reduce(es.elapsed_time(ee) / n, "max")

        def step_graphs(fn):
            """Runs exactly k steps of ``fn`` (cycling the layers) as graphs
            of ``chunk`` steps plus one graph of the remainder, the way the
            headline runs its steps and a decoder replays one graph per
            token over its layers; every graph is captured and uploaded
            before it is timed."""
            made = {}

            def graph(n):
                if n not in made:
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=self.stream):
                        for i in range(n):
                            fn(i % self.layers)
                    upload_graph(gr)
                    made[n] = gr
                return made[n]

            def run(k):
                for _ in range(k // self.chunk):
                    graph(self.chunk).replay()
                if k % self.chunk:
                    graph(k % self.chunk).replay()

            def prepare(k):
                if k // self.chunk:
                    graph(self.chunk)
                if k % self.chunk:
                    graph(k % self.chunk)

            return run, prepare

        def timed_graphs(fn, n):
            run, prepare = step_graphs(fn)
            prepare(3)
            prepare(n)
            run(3)
            torch.cuda.synchronize()
            dist.barrier()
            es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            es.record()
            run(n)
            ee.record()
            torch.cuda.synchronize()
            dist.barrier()
            return dist.reduce(es.elapsed_time(ee) / n, "max")

        with torch.cuda.stream(self.stream):
            eager_ms = timed(lambda i: one(i % self.layers), steps)
            graph_ms, err = None, None
            try:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=self.stream):
                    one(0)
                del gr
                torch.cuda.synchronize()
                ok = 1.0
            except RuntimeError as exc:  # capture of pinned copies refused
                ok, err = 0.0, str(exc).splitlines()[0][:200]
                torch.cuda.synchronize()
            if dist.reduce(ok, "sum") == dist.world:
                graph_ms = timed_graphs(one, steps)
            zc_ms = timed_graphs(one_zero_copy, steps)
            # For comparison: one graph per step (a caller that captures a
            # single layer's step and replays it per call).
            zc_graphs = []
            for layer in range(self.layers):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=self.stream):
                    one_zero_copy(layer)
                upload_graph(gr)
                zc_graphs.append(gr)
            zc_single_ms = timed(lambda i: zc_graphs[i % self.layers].replay(), steps)
            # The zero-copy result must equal the copy path's.
            one(0)
            torch.cuda.synchronize()
            ref = hout.clone()
            one_zero_copy(0)
            torch.cuda.synchronize()
            zc_equal = bool(torch.equal(ref, hout))
        h2d = hqkv.numel() * 2
        return {"eager_ms": eager_ms, "graph_ms": graph_ms, "graph_error": err,
                "zero_copy_graph_ms": zc_ms, "zero_copy_equal": zc_equal,
                "zero_copy_single_graph_ms": zc_single_ms,
                "h2d": h2d, "d2h": hout.numel() * 2, "launches_per_step": 1 + self.launches_per_step}


class AffineBench(AttentionBench):
    """The reference's alternative representation, affine_group16 (INT8
    codes with an FP16 scale and bias per page, head and 16-dim group; no
    centres), on the same workload: every completed page quantised by the
    bulk affine quantiser, the last TAIL_PAGES pages read as plain FP16 from
    the dense cache (the reference's exact-segments run of this
    representation, scripts/benchmark_flashinfer_page_affine_int8.py:528-602)."""

    def __init__(self, lengths, layers: int, split: int, seed: int, warps: int = 4):
        from pagegauge_b200 import scheduler
        from pagegauge_b200.cache import synthetic_dense_cache
        from pagegauge_b200.decode import PageGaugeDecode, split_tables
        from pagegauge_b200.quantize import quantize_pages

        self.lengths = lengths
        self.layers = max(1, layers)
        self.fused, self.cluster = False, 0
        pages = [-(-n // PAGE) for n in lengths]
        o_ptr, o_idx, e_ptr, e_idx = split_tables(pages, TAIL_PAGES)
        self.data = []
        self.q = None
        for layer in range(self.layers):
            qi, dk, dv = synthetic_dense_cache(lengths, seed=seed + layer, device="cuda")
            kc, kb, ks, _ = quantize_pages(dk)
            vc, vb, vs, _ = quantize_pages(dv)
            self.data.append((kc, vc, ks, vs, dk, dv, (kb, vb)))
            self.q = qi if self.q is None else self.q
        torch.cuda.synchronize()
        if split < 0:
            split = scheduler.lookup(len(lengths), max(lengths), representation="affine_group16")
        last = torch.tensor([(n - 1) % PAGE + 1 for n in lengths], dtype=torch.int32, device="cuda")
        self.ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.dec = PageGaugeDecode(self.ws, warps_per_cta=warps)
        self.dec.plan(o_ptr, torch.from_numpy(o_idx).cuda(), e_ptr, torch.from_numpy(e_idx).cuda(),
                      last, HQ, HKV, old_split_pages=split, exact_split_pages=0)
        self.plan = self.dec.work_plan
        self.out = torch.empty_like(self.q)
        old_pages = [int(o_ptr[r + 1] - o_ptr[r]) for r in range(len(lengths))]
        # codes (K+V) + 64 bytes of group scales/biases per (page, head) +
        # the FP16 tail
        self.nbytes = sum(op * HKV * (2 * PAGE * DIM + 64) + 2 * 2 * (n - op * PAGE) * HKV * DIM
                          for op, n in zip(old_pages, lengths))
        self.launches_per_step = 1 if (self.plan.single and self.plan.num_items) else 2
        self.stream = torch.cuda.Stream()
        self.chunk = 8 * self.layers

    def layer_tensors(self, layer: int):
        return self.data[layer]

    def step(self, layer: int, q=None, out=None):
        kc, vc, ks, vs, dk, dv, affine = self.data[layer]
        self.dec.run(self.q if q is None else q, kc, vc, ks, vs, dk, dv, None,
                     out=self.out if out is None else out, affine_bias=affine)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ------------------------------------------------------------ append bench
def measure_append(dist: Dist, batch: int = 8, layers: int = 32, samples: int = 100) -> dict:
    """The fused-append benchmark: one decode step's fused RoPE + centred append +
    page finalisation for B=8 requests in each of 32 layers (one launch per
    layer), half of the requests at the last token of a page (position %
    16 == 15, so their page is finalised to INT8 in the same launch), the
    other half mid-page; against the fused RoPE + FP16 append comparator
    on the same inputs.  Cache-neutral: a 256 MiB scrub before every sample;
    samples alternate A/B then B/A; p50."""
    from pagegauge_b200.cache import rope_tables
    from pagegauge_b200.runtime import load_append_extension

    ext = load_append_extension()
    ppr, ring = 64, TAIL_PAGES
    positions = torch.tensor([16 * (4 * r + 3) + (15 if r % 2 == 0 else 7) for r in range(batch)],
                             dtype=torch.int32, device="cuda")
    closes = int(((positions % 16) == 15).sum())
    cos, sin = rope_tables(ppr * PAGE, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(SEED + 3)
    per = []
    for _ in range(layers):
        offset = torch.randn(HKV, DIM, generator=g, device="cuda")
        d = dict(
            q=torch.randn(batch, HQ, DIM, generator=g, device="cuda").half(),
            k=(torch.randn(batch, HKV, DIM, generator=g, device="cuda") + offset).half(),
            v=(torch.randn(batch, HKV, DIM, generator=g, device="cuda") + 0.5 * offset).half(),
            kc=offset.half().expand(batch, HKV, DIM).contiguous(),
            vc=(0.5 * offset).half().expand(batch, HKV, DIM).contiguous(),
            rq=torch.empty(batch, HQ, DIM, dtype=torch.float16, device="cuda"),
            ek=torch.zeros(batch * ring, PAGE, HKV, DIM, dtype=torch.float16, device="cuda"),
            codes_k=torch.zeros(batch * ppr, PAGE, HKV, DIM, dtype=torch.int8, device="cuda"),
            sk=torch.zeros(batch * ppr, HKV, dtype=torch.float16, device="cuda"),
            fk=torch.zeros(batch * ppr, PAGE, HKV, DIM, dtype=torch.float16, device="cuda"),
        )
        d["ev"] = torch.zeros_like(d["ek"])
        d["codes_v"] = torch.zeros_like(d["codes_k"])
        d["sv"] = torch.zeros_like(d["sk"])
        d["fv"] = torch.zeros_like(d["fk"])
        d["rq16"] = torch.empty_like(d["rq"])
        per.append(d)

    def gauge():
        for d in per:
            ext.rope_append_page_gauge_batched(d["q"], d["k"], d["v"], cos, sin, positions, d["kc"],
                                               d["vc"], d["rq"], d["ek"], d["ev"], d["codes_k"],
                                               d["codes_v"], d["sk"], d["sv"], 0)

    def fp16():
        for d in per:
            ext.rope_append_fp16_batched(d["q"], d["k"], d["v"], cos, sin, positions, d["rq16"],
                                         d["fk"], d["fv"])

    stream = torch.cuda.Stream()
    graphs = {}
    with torch.cuda.stream(stream):
        for name, fn in (("gauge", gauge), ("fp16", fp16)):
            fn()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                fn()
            graphs[name] = gr
        torch.cuda.synchronize()
        scrub = torch.zeros(256 << 18, dtype=torch.int32, device="cuda")
        times = {"gauge": [], "fp16": []}
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        dist.barrier()
        for i in range(samples):
            order = ("gauge", "fp16") if i % 2 == 0 else ("fp16", "gauge")
            for name in order:
                scrub.add_(1)
                ev[0].record()
                graphs[name].replay()
                ev[1].record()
                ev[1].synchronize()
                times[name].append(ev[0].elapsed_time(ev[1]))
        hot = {}
        for name in ("gauge", "fp16"):
            graphs[name].replay()
            torch.cuda.synchronize()
            ev[0].record()
            for _ in range(50):
                graphs[name].replay()
            ev[1].record()
            ev[1].synchronize()
            hot[name] = ev[0].elapsed_time(ev[1]) / 50
        dist.barrier()
    del graphs
    p50 = {k: dist.reduce(statistics.median(v), "max") for k, v in times.items()}
    hot = {k: dist.reduce(v, "max") for k, v in hot.items()}
    # Algorithmic bytes per layer: q read + rotated q write, k/v read,
    # centres, one cos/sin row per request, ring writes, and per closed page
    # the ring page re-read, the codes write and the two scales.
    b = batch
    per_layer = (2 * b * HQ * DIM * 2 + 2 * b * HKV * DIM * 2 + 2 * b * HKV * DIM * 2
                 + 2 * b * DIM * 2 + 2 * b * HKV * DIM * 2
                 + closes * HKV * (2 * PAGE * DIM * 2 + 2 * PAGE * DIM + 2 * 2))
    return {
        "batch": batch, "layers": layers, "closing_requests": closes,
        "us_per_step": p50["gauge"] * 1e3, "us_per_layer": p50["gauge"] * 1e3 / layers,
        "fp16_append_us_per_step": p50["fp16"] * 1e3,
        "increment_us_per_step": (p50["gauge"] - p50["fp16"]) * 1e3,
        "hot_us_per_step": hot["gauge"] * 1e3, "hot_fp16_us_per_step": hot["fp16"] * 1e3,
        "algorithmic_bytes_per_layer": per_layer,
        "achieved_gbs": per_layer * layers / (p50["gauge"] * 1e-3) / 1e9,
        "timing": f"p50 of {samples} cache-neutral samples (256 MiB scrub before each), "
                  "A/B then B/A order; one CUDA graph of 32 launches per sample",
    }


# ---------------------------------------------------------- decoder bench
def decoder_bytes(dec, batch: int) -> int:
    """HBM bytes one decode step reads on this rank: every local weight
    (the embedding only for the batch's rows) plus the PageGauge caches of
    this rank's KV heads (INT8 codes + scales of the old pages, the FP16
    exact window)."""
    w = dec.w
    total = sum(t.numel() * 2 for lw in w.layers
                for t in (lw.attn_norm, lw.qkv, lw.o, lw.mlp_norm, lw.gate_up, lw.down))
    total += w.lm_head.numel() * 2 + w.final_norm.numel() * 2 + batch * w.embed.shape[1] * 2
    old, exact = [], []
    from pagegauge_b200.decoder import page_tables
    o_ptr, _, _, _ = page_tables(dec.host_positions, dec.capacity_pages, dec.ring_pages,
                                 dec.sink_pages, dec.suffix_pages, dec.initial_pages)
    for r, p in enumerate(dec.host_positions):
        n_old = int(o_ptr[r + 1] - o_ptr[r])
        old.append(n_old * PAGE)
        exact.append(int(p) + 1 - n_old * PAGE)
    return total + dec.cfg.layers * algorithmic_bytes(old, exact, hkv=dec.hkv)


def parse_policy(text: str) -> tuple[int, int, int]:
    """'S4/A0/T768' -> (sink pages, suffix pages, ring pages)."""
    parts = dict((p[0].upper(), int(p[1:])) for p in text.split("/"))
    if parts.get("T", 256) % PAGE:
        raise ValueError("the tail must be whole pages")
    return parts.get("S", 0), parts.get("A", 0), parts.get("T", 256) // PAGE


def measure_decoder(dist: Dist, batch: int, context: int = 16384, steps: int = 16,
                    seed: int = 20261004, gemm: str = "auto", policy: str = "S0/A0/T256",
                    tp_reduce: str = "peer") -> dict:
    """The benchmark decoder: Mistral-7B-shaped random-init FP16 decoder,
    prompt of ``context`` random tokens prefilled into PageGauge caches, one
    eager warm-up decode step, then ``steps`` greedy decode steps (CUDA
    graphs prepared beforehand), tensor-parallel over the ranks."""
    from pagegauge_b200.decoder import (DecoderConfig, PageGaugeDecoder, TensorParallel,
                                        random_decoder_weights)
    from pagegauge_b200.runtime import read_device_error

    world = dist.world
    rank = int(os.environ.get("RANK", "0"))
    pg = dist.dist.group.WORLD if dist.dist is not None else None
    cfg = DecoderConfig.mistral_7b_shaped()
    t0 = time.perf_counter()
    w = random_decoder_weights(cfg, seed, device="cuda", tp=TensorParallel.of(cfg, rank, world))
    sink, suffix, ring = parse_policy(policy)
    dec = PageGaugeDecoder(w, batch, max_context=context + 4 * steps + 32, process_group=pg,
                           gemm=gemm, ring_pages=ring, sink_pages=sink, suffix_pages=suffix,
                           tp_reduce=tp_reduce)
    prompt = torch.randint(0, cfg.vocab, (batch, context),
                           generator=torch.Generator().manual_seed(seed + batch))
    dec.prefill(prompt.cuda())
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    dec.step(use_graph=True)  # eager warm-up step (cuBLAS / NCCL on the decode stream)
    dec.prepare(steps)
    nbytes = decoder_bytes(dec, batch)
    torch.cuda.synchronize()
    dist.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.nvtx.range_push("pg_timed")
    ev[0].record(dec.stream)
    for _ in range(steps):
        dec.step()
    ev[1].record(dec.stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    dist.barrier()
    ms = dist.reduce(ev[0].elapsed_time(ev[1]) / steps, "max")
    # End to end: every step's tokens come back to pinned host memory and the
    # host waits for them before launching the next step.
    dec.prepare(steps)
    host = torch.empty(batch, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    dist.barrier()
    t1 = time.perf_counter()
    for _ in range(steps):
        dec.step()
        host.copy_(dec.tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_s = dist.reduce((time.perf_counter() - t1) / steps, "max")
    achieved = nbytes / (ms * 1e-3) / 1e9
    peak, _ = peak_hbm()
    out = {
        "batch": batch, "context": context, "tp": world, "steps": steps,
        "tokens_per_s": round(batch / (ms * 1e-3), 2), "ms_per_step": ms,
        "kernel_launches_per_step": dec.launches_per_step(),
        "e2e_tokens_per_s": round(batch / e2e_s, 2),
        "hbm_bytes_per_step_per_rank": nbytes, "achieved_gbs_per_rank": round(achieved, 1),
        "roofline_frac": round(achieved / peak, 4), "prefill_s": round(prefill_s, 2),
        "replans_in_timing": 0, "params": cfg.parameter_count(), "gemm": dec.gemm_impl,
        "exact_policy": policy,
        "tp_reduce": (None if world == 1 else ("peer" if dec.tpx is not None else "nccl")),
        "device_guard": read_device_error(),
    }
    dec.close()
    del dec, w
    torch.cuda.empty_cache()
    return out


def run_decoder(args, dist: Dist, local: int) -> None:
    rank = int(os.environ.get("RANK", "0"))
    clocks = ClockSampler(local)
    batches = args.decoder_batch or [32]
    results = {}
    with clocks:
        results[batches[0]] = measure_decoder(dist, batches[0], steps=args.decoder_steps,
                                              gemm=args.decoder_gemm, policy=args.decoder_policy,
                                              tp_reduce=args.decoder_tp_reduce)
    for b in batches[1:]:
        results[b] = measure_decoder(dist, b, steps=args.decoder_steps, gemm=args.decoder_gemm,
                                     policy=args.decoder_policy, tp_reduce=args.decoder_tp_reduce)
    b32 = results[batches[0]]
    peak, peak_src = peak_hbm()
    if rank == 0:
        line = {
            "metric": f"decoder tokens/s (Mistral-7B-shaped, B={batches[0]}, ctx 16384)",
            "value": b32["tokens_per_s"], "unit": "tokens/s", "n_gpus": dist.world,
            "steps": b32["steps"], "warmup": 1, "ms_per_step": b32["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 weights/activations, int8 page-gauge KV",
            "data": "synthetic (random-init N(0,0.02) weights, random prompt tokens)",
            "config": {"workload": "decoder", "layers": 32, "hidden": 4096, "heads": 32,
                       "kv_heads": 8, "ffn": 14336, "vocab": 32768, "context": 16384,
                       "decode_tokens": 16, "parallelism": f"tp{dist.world}"},
            "roofline": {"bound": "hbm", "achieved": b32["achieved_gbs_per_rank"], "peak": peak,
                         "unit": "GB/s", "frac": b32["roofline_frac"], "traffic": None,
                         "peak_source": peak_src, "kernel": "whole decode step"},
            "e2e": {"value": b32["e2e_tokens_per_s"], "unit": "tokens/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 8 * batches[0]},
            "clocks": clocks.summary(),
            "workloads": {f"decoder_b{b}": r for b, r in results.items()},
        }
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------ projections
def run_gemm(args) -> None:
    """The decoder's projection GEMMs alone at its one-row shapes (Mistral-7B
    layer: qkv, o + residual, gate|up + SiLU*up, down + residual; the LM
    head), each streamed from enough weight copies to exceed the L2 and
    replayed back to back in a CUDA graph (PDL between launches); a
    secondary measurement of the weight-streaming kernel, not a headline."""
    from pagegauge_b200.gemm import RESIDUAL, SILU_MUL, STORE, PackedWeight, SkinnyGemm

    batch = 1
    peak, peak_src = peak_hbm()
    shapes = {"qkv": (6144, 4096, STORE), "o": (4096, 4096, RESIDUAL),
              "gate_up": (28672, 4096, SILU_MUL), "down": (4096, 14336, RESIDUAL),
              "lm_head": (32768, 4096, STORE)}
    g = torch.Generator(device="cuda").manual_seed(SEED)
    results, total_bytes, total_us = {}, 0, 0.0
    for name, (n, k, mode) in shapes.items():
        copies = max(2, int(400e6 // (n * k * 2)) + 1)
        ws = [PackedWeight((torch.randn(n, k, generator=g, device="cuda") * 0.02).half(), mode)
              for _ in range(copies)]
        x = torch.randn(batch, k, generator=g, device="cuda").half()
        res = torch.zeros(batch, n, device="cuda").half()
        out = torch.empty(batch, n // 2 if mode == SILU_MUL else n, device="cuda").half()
        gemm = SkinnyGemm("cuda")
        gemm.reserve(n, k, batch, mode)
        stream = torch.cuda.Stream()
        torch.cuda.nvtx.range_push(f"gemm_{name}")

        def run(w):
            if mode == RESIDUAL:
                gemm(x, w, mode=mode, residual=res)
            else:
                gemm(x, w, out=out, mode=mode)

        with torch.cuda.stream(stream):
            for w in ws:
                run(w)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(4 * copies):
                    run(ws[i % copies])
            for _ in range(max(args.warmup, 3) // 3 + 1):
                graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 5
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        us = e0.elapsed_time(e1) * 1e3 / (reps * 4 * copies)
        nbytes = n * k * 2
        results[name] = {"n": n, "k": k, "us": round(us, 3),
                         "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                         "roofline_frac": round(nbytes / (us * 1e-6) / 1e9 / peak, 4)}
        total_bytes += nbytes
        total_us += us
        del graph, ws
        torch.cuda.empty_cache()
    value = total_bytes / (total_us * 1e-6) / 1e9
    print(json.dumps({
        "metric": "decoder projection GEMMs, weight GB/s (B=1)", "value": round(value, 1),
        "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "dtype": "fp16 in, fp32 accumulate",
        "data": "synthetic random N(0,0.02) weights",
        "config": {"workload": "gemm", "batch": batch, "shapes": list(shapes)},
        "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / peak, 4), "peak_source": peak_src,
                     "kernel": "pg_skinny_gemm_kernel"},
        "workloads": results}), flush=True)


# -------------------------------------------------------------------- main
def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local))
    dist = Dist(world)

    from pagegauge_b200.runtime import read_device_error

    if args.workload == "decoder":
        run_decoder(args, dist, local)
        if world > 1:
            dist.barrier()
            dist.dist.destroy_process_group()
        return
    if args.workload == "append":
        # configs[3] alone: the fused append step (B=8, 32 layers) and the
        # FP16 comparator, as in the default line's workloads.
        app = measure_append(dist)
        if rank == 0:
            print(json.dumps({
                "metric": "fused append step us (B=8, 32 layers)", "value": app["us_per_step"],
                "unit": "us", "n_gpus": world, "higher_is_better": False,
                "dtype": "fp16 RoPE, fp32 centring, int8 codes", "data": "synthetic",
                "config": {"workload": "append", "batch": 8, "layers": 32},
                "workloads": {"append_b8_32l": app}}), flush=True)
        if world > 1:
            dist.barrier()
            dist.dist.destroy_process_group()
        return
    if args.workload == "gemm":
        if rank == 0:
            run_gemm(args)
        if world > 1:
            dist.barrier()
            dist.dist.destroy_process_group()
        return
    peak, peak_src = peak_hbm()
    lengths, glob, shards = workload_lengths(args.workload, world, rank)
    clocks = ClockSampler(local)
    clocks.start()  # covers every measurement below
    secondary = not args.only and args.workload == "b1_49k"
    workloads = {}
    # The memory-bound secondary workloads run first: the headline's timed
    # steps then find the GPU at its working clocks rather than ramping up
    # from idle (a 20-step run lasts well under a millisecond).
    if secondary:
        workloads["b8_ragged"] = measure_b8_sharded(args, dist, rank, peak)
        app = measure_append(dist)
        if world == 1:
            # The append's share of a decode step: against the B8 attention
            # step of the same 8 requests on one GPU (first seed).
            attn_layer_us = workloads["b8_ragged"]["per_seed"][0]["us_per_step"]
            app["attention_us_per_layer_b8"] = attn_layer_us
            app["pct_of_attention_step"] = round(100 * app["us_per_layer"] / attn_layer_us, 2)
            app["increment_pct_of_attention_step"] = round(
                100 * app["increment_us_per_step"] / app["layers"] / attn_layer_us, 2)
        app["scaling"] = "weak (replicas)"
        workloads["append_b8_32l"] = app
        aff = AffineBench(lengths, args.layers, args.split, seed=SEED + 1000 * rank + 900,
                          warps=args.warps)
        aff.capture()
        aff_steps = max(200, args.steps // 10)
        aff_ms = aff.time_steps(aff_steps, args.warmup, dist)
        aff_kms = dist.reduce(aff.kernel_ms(aff_steps), "max")
        workloads["affine_group16_" + args.workload] = {
            "metric": f"decode-attn HBM GB/s (affine_group16, {args.workload})", "unit": "GB/s",
            "value": round(dist.reduce(float(aff.nbytes), "sum") / (aff_ms * 1e-3) / 1e9, 2),
            "us_per_step": aff_ms * 1e3, "steps": aff_steps, "kernel_us": aff_kms * 1e3,
            "roofline_frac": round(aff.nbytes / (aff_kms * 1e-3) / 1e9 / peak, 4),
            "algorithmic_bytes_per_step_per_rank": aff.nbytes,
            "split_pages": aff.plan.split_pages[0], "work_items": aff.plan.num_items,
            "scaling": "weak (replicas)",
            "note": "the reference's rejected representation, same kernel family; "
                    "page_gauge is the headline",
        }
        del aff
        torch.cuda.empty_cache()

    bench = AttentionBench(lengths, args.layers, args.split, args.merge == "fused",
                           seed=SEED + 1000 * rank, warps=args.warps,
                           cluster=args.cluster if args.merge == "cluster" else 0)
    bench.capture()
    ms = bench.time_steps(args.steps, args.warmup, dist)
    total_bytes = dist.reduce(float(bench.nbytes), "sum")
    value = total_bytes / (ms * 1e-3) / 1e9
    kernel_ms = dist.reduce(bench.kernel_ms(args.steps), "max")
    achieved = bench.nbytes / (kernel_ms * 1e-3) / 1e9
    e2e = bench.e2e(args.steps, dist)
    graphs_of = (f"CUDA graphs of {bench.chunk} public-API steps ({bench.layers} layer caches "
                 f"cycled) and one of the remainder, each step with its own host transfers")
    e2e_ms = e2e["graph_ms"] if e2e["graph_ms"] is not None else e2e["eager_ms"]
    e2e_mode = (graphs_of + ": pinned H2D copy of q|k|v, append, decode, D2H copy of the output"
                if e2e["graph_ms"] is not None else "eager public-API calls")
    if e2e["zero_copy_equal"] and e2e["zero_copy_graph_ms"] < e2e_ms:
        e2e_ms = e2e["zero_copy_graph_ms"]
        e2e_mode = (graphs_of + ": the append reads q|k|v from pinned host memory and the "
                    "decode writes the output to pinned host memory (zero copy)")
    plan_info = {"split_pages": bench.plan.split_pages[0], "work_items": bench.plan.num_items,
                 "launches_per_step": bench.launches_per_step}
    del bench
    torch.cuda.empty_cache()

    if secondary:
        for b in (1, 32):
            d = measure_decoder(dist, b, steps=args.decoder_steps, gemm=args.decoder_gemm,
                                policy=args.decoder_policy, tp_reduce=args.decoder_tp_reduce)
            d["scaling"] = f"strong (tensor parallel over {world} GPU(s))"
            workloads[f"decoder_b{b}"] = d
    clocks.stop()
    err = read_device_error()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(lengths[:1])
        if "decoder_b1" in workloads:
            workloads["decoder_b1"]["cpu_baseline"] = decoder_cpu_baseline()

    if rank == 0:
        line = {
            "metric": f"decode-attn HBM GB/s ({args.workload})",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "us_per_step": ms * 1e3,
            "higher_is_better": True,
            "scaling": "weak" if shards is None else "strong", "vs_baseline": None,
            "dtype": "int8 codes + fp16 tail, fp16 mma / fp32 softmax",
            "data": "synthetic (seeded; K=RoPE(N(mu,1)), mu~N(0,2); V,Q~N(0,1))",
            "config": workload_config(args, world),
            "plan": plan_info,
            "algorithmic_bytes_per_step": workload_bytes(lengths),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic(args.workload), "peak_source": peak_src,
                         "kernel": "pg_decode_split_kernel", "kernel_us": kernel_ms * 1e3},
            "gpu_launches": plan_info["launches_per_step"] * args.steps,
            "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "us_per_step": e2e_ms * 1e3,
                    "mode": e2e_mode,
                    "copy_graph_us_per_step": (None if e2e["graph_ms"] is None
                                               else e2e["graph_ms"] * 1e3),
                    "zero_copy_us_per_step": e2e["zero_copy_graph_ms"] * 1e3,
                    "zero_copy_one_graph_per_step_us": e2e["zero_copy_single_graph_ms"] * 1e3,
                    "zero_copy_equal": e2e["zero_copy_equal"],
                    "eager_value": round(total_bytes / (e2e["eager_ms"] * 1e-3) / 1e9, 2),
                    "eager_us_per_step": e2e["eager_ms"] * 1e3,
                    "graph_error": e2e["graph_error"],
                    "launches_per_step": e2e["launches_per_step"]},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "device_guard": err,
            "workloads": workloads,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.dist.destroy_process_group()


def measure_b8_sharded(args, dist: Dist, rank: int, peak: float) -> dict:
    """the 8 ragged requests of each seed, sharded over the ranks
    by longest-first bin packing (strong scaling: the same 8 requests at
    every N, no data-path collective).  Per seed: max-over-ranks step time,
    aggregate GB/s, the kernel's roofline fraction and the per-rank byte
    imbalance (max / mean)."""
    from pagegauge_b200.shard import plan_shards

    world = dist.world
    steps = max(200, args.steps // 10)
    per_seed = []
    for seed in SEEDS:
        glob = global_lengths("b8_ragged", seed)
        plan = plan_shards(glob, world, kv_heads=HKV)
        shards, loads = plan["requests"], plan["rank_bytes"]
        mine = [glob[i] for i in shards[rank]]
        h0, h1 = plan["heads"][rank]
        hkv = h1 - h0
        sharding = ("requests (longest-first bin packing on decode bytes)"
                    if plan["mode"] == "requests"
                    else f"KV heads ({hkv} of {HKV} per GPU, all requests)")
        if mine:
            b8 = AttentionBench(mine, args.layers, -1, False, seed=seed, hkv=hkv)
            b8.capture()
            my_bytes = b8.nbytes
            b8_ms = b8.time_steps(steps, args.warmup, dist)
            b8_kms = dist.reduce(b8.kernel_ms(steps), "max")
            split, items = b8.plan.split_pages[0], b8.plan.num_items
            del b8
            torch.cuda.empty_cache()
        else:  # more ranks than requests: this rank only joins the collectives
            my_bytes, split, items = 0, 0, 0
            dist.barrier()  # the two barriers and the reduce of time_steps
            dist.barrier()
            b8_ms = dist.reduce(0.0, "max")
            b8_kms = dist.reduce(0.0, "max")
        total = dist.reduce(float(my_bytes), "sum")
        per_seed.append({
            "seed": seed, "lengths": glob, "shards": shards, "value_gbs": round(total / (b8_ms * 1e-3) / 1e9, 2),
            "us_per_step": b8_ms * 1e3, "kernel_us": b8_kms * 1e3,
            "kernel_frac_of_peak": round(max(loads) / (b8_kms * 1e-3) / 1e9 / peak, 4),
            "algorithmic_bytes_per_step": int(total), "rank_bytes": loads, "sharding": sharding,
            "imbalance": round(max(loads) / (sum(loads) / len(loads)), 4),
            "split_pages_rank0": split, "work_items_rank0": items,
        })
    tot_bytes = sum(x["algorithmic_bytes_per_step"] for x in per_seed)
    tot_us = sum(x["us_per_step"] for x in per_seed)
    return {"metric": "decode-attn HBM GB/s (b8_ragged, 3 seeds)", "unit": "GB/s",
            "value": round(tot_bytes / (tot_us * 1e-6) / 1e9, 2),
            "us_per_step_mean": tot_us / len(per_seed), "steps": steps,
            "scaling": f"strong (the same 8 requests over {world} GPU(s), sharded by request "
                       f"or by KV head, whichever balances the bytes)",
            "per_seed": per_seed}


if __name__ == "__main__":
    main()
