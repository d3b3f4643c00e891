"""Split-KV scheduler: pick pages per work item (``num_splits`` =
ceil(pages / split)) per (batch, context) bucket from measured timings.

The reference froze one ``fixed_split_size`` per method from a pilot sweep
over {auto, 64, 128, 256, 512} pages, keeping the cache-neutral p50 argmin
(scripts/run_page_gauge_validation.py:277-316, B1/49K at :374-416).  Here
the sweep covers num_splits 1..64 per KV head (and the one-wave
heuristic), each candidate timed on the GPU as a decoder runs it (back to
back over caches larger than the L2; ``--mode burst`` times single decodes
behind a 256 MiB scrub instead), and the argmin is stored per (batch,
half-octave context) bucket in ``split_table.json`` next to this file.

    python -m pagegauge_b200.scheduler --sweep [--batch 1 --context 49152] [--kv-heads 8 1]
        [--representation affine_group16]
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
from pathlib import Path

TABLE_PATH = Path(__file__).resolve().parent / "split_table.json"
PAGE = 16


REPRESENTATIONS = ("page_gauge", "affine_group16")


def bucket(batch: int, context: int, kv_heads: int = 8,
           representation: str = "page_gauge") -> str:
    """Batch exact, context rounded down to a half octave (2^k or 1.5 * 2^k,
    >= 1024): bucket 2^k covers [2^k, 1.5 * 2^k), bucket 1.5 * 2^k covers
    [1.5 * 2^k, 2^(k+1)); KV heads other than 8 (a tensor-parallel or
    head-sharded rank) and the affine_group16 representation (a different
    kernel instantiation) get their own entries."""
    if representation not in REPRESENTATIONS:
        raise ValueError(f"unknown representation {representation!r}")
    k = max(10, int(math.floor(math.log2(max(context, 1)))))
    c = 1 << k
    if k >= 11 and context >= c + c // 2:
        c += c // 2
    return (f"b{batch}_c{c}" + ("" if kv_heads == 8 else f"_h{kv_heads}")
            + ("" if representation == "page_gauge" else "_affine"))


def load_table(path: Path = TABLE_PATH) -> dict:
    if path.is_file():
        return json.loads(path.read_text())
    return {"entries": {}}


def lookup(batch: int, context: int, path: Path = TABLE_PATH, kv_heads: int = 8,
           representation: str = "page_gauge") -> int:
    """Pages per work item for this shape; 0 (the one-wave heuristic) when
    the bucket was never measured.  With fewer than 8 KV heads and no entry
    of its own, the 8-head entry scaled by kv_heads / 8 (each head split
    finer, so the work list still fills about one wave); affine_group16
    without an entry of its own takes the page_gauge entry."""
    entries = load_table(path)["entries"]
    for rep in dict.fromkeys((representation, "page_gauge")):
        entry = entries.get(bucket(batch, context, kv_heads, rep))
        if entry:
            return int(entry["split_pages"])
        entry = entries.get(bucket(batch, context, 8, rep))
        if entry:
            return max(1, int(entry["split_pages"]) * kv_heads // 8)
    return 0


MAX_SPLIT_PAGES = 128  # the planner's cap: 32 pages per warp at 4 warps per CTA


def candidates(old_pages_per_request: int, max_split: int = MAX_SPLIT_PAGES) -> list[int]:
    """Split sizes giving num_splits in 1..64 per (request, head), plus 0
    for the one-wave heuristic; sizes above the planner's cap would all
    run as the cap, so the cap stands for them."""
    out = {0}
    for splits in (1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64):
        out.add(min(max_split, max(1, math.ceil(old_pages_per_request / splits))))
    return sorted(out)


def record(batch: int, context: int, results: dict[int, float], path: Path = TABLE_PATH,
           meta: dict | None = None, kv_heads: int = 8,
           representation: str = "page_gauge") -> int:
    """Store the argmin of {split_pages: p50 microseconds}."""
    best = min(results, key=results.get)
    table = load_table(path)
    table["entries"][bucket(batch, context, kv_heads, representation)] = {
        "split_pages": int(best), "p50_us": results[best],
        "candidates_us": {str(k): v for k, v in sorted(results.items())}, **(meta or {})}
    path.write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    return best


def sweep(batch: int, context: int, repeats: int = 30, seeds=(20261001, 20261002, 20261003),
          write: bool = True, path: Path = TABLE_PATH, lengths: list[int] | None = None,
          burst: int = 16, mode: str = "steady", layers: int = 4,
          kv_heads: int = 8, representation: str = "page_gauge") -> dict[int, float]:
    """Time every candidate split on the current GPU and record the winner.

    ``mode="steady"`` (the default): ``layers`` caches of the shape (more
    bytes than the 126 MB L2 together) decoded back to back in a CUDA
    graph of ``8 * layers`` steps cycling the caches, as a decoder runs its
    layers (each launch overlaps its start-up with the previous step's tail
    through programmatic dependent launch); a sample is one replay between
    CUDA events divided by its steps.  ``mode="burst"``: each candidate's
    decode behind a 256 MiB scrub in one graph, ``burst`` replays minus the
    same burst of a scrub-only graph (every step starts from a cold L2 and
    an idle GPU).  The p50 over ``repeats`` samples per seed is averaged
    over the seeds.  ``lengths`` (default ``[context] * batch``) gives
    ragged batches; the table bucket is (batch, max length)."""
    import torch

    if mode == "steady":
        return _sweep_steady(batch, context, repeats, seeds, write, path, lengths, layers,
                             kv_heads, representation)
    if kv_heads != 8 or representation != "page_gauge":
        raise ValueError("the burst mode sweeps 8-head page_gauge caches only")
    from .cache import build_gauge_cache, synthetic_dense_cache
    from .decode import PageGaugeDecode

    lengths = list(lengths) if lengths is not None else [context] * batch
    batch, context = len(lengths), max(lengths)
    scrub = torch.zeros(256 << 18, dtype=torch.int32, device="cuda")  # 256 MiB
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        scrub.add_(1)
        scrub_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(scrub_graph, stream=stream):
            scrub.add_(1)
    torch.cuda.synchronize()

    def burst_us(graph) -> float:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(burst):
            graph.replay()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) * 1e3

    results: dict[int, list[float]] = {}
    for seed in seeds:
        q, dk, dv = synthetic_dense_cache(lengths, seed=seed, device="cuda")
        cache, tables = build_gauge_cache(dk, dv, lengths)
        del dk, dv
        old_pages = max(t // PAGE for t in tables.old_tokens)
        out = torch.empty_like(q)
        for split in candidates(old_pages):
            dec = PageGaugeDecode(ws)
            dec.plan(tables.old_indptr, tables.old_indices, tables.exact_indptr,
                     tables.exact_indices, tables.exact_last_page_len, 32, 8,
                     old_split_pages=split)

            def run():
                dec.run(q, cache.key_codes, cache.value_codes, cache.key_scales,
                        cache.value_scales, cache.exact_key, cache.exact_value,
                        cache.value_center, out=out)

            with torch.cuda.stream(stream):
                for _ in range(3):
                    run()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    scrub.add_(1)
                    run()
                for _ in range(3):
                    graph.replay()
                times = []
                for _ in range(repeats):
                    both = burst_us(graph)
                    only = burst_us(scrub_graph)
                    times.append((both - only) / burst)
            torch.cuda.synchronize()
            del graph
            results.setdefault(split, []).append(statistics.median(times))
        del cache
    p50 = {k: statistics.fmean(v) for k, v in results.items()}
    if write:
        record(batch, context, p50, path=path,
               meta={"gpu": torch.cuda.get_device_name(), "repeats": repeats,
                     "seeds": list(seeds), "lengths": lengths,
                     "burst": burst,
                     "mode": "cache-neutral: CUDA graph of scrub + decode, minus scrub alone"})
    return p50


def refinements(best: int, measured) -> list[int]:
    """Split sizes within +-20 % of the coarse winner not yet measured (the
    coarse candidates are num_splits steps, up to 15 % apart)."""
    if best <= 0:
        return []
    out = {max(1, round(best * f)) for f in (0.8, 0.85, 0.9, 0.95, 1.05, 1.1, 1.15, 1.2)}
    return sorted(out - set(measured))


def _layer_setup(lengths, seed: int, kv_heads: int, representation: str):
    """One layer's cache for the steady sweep: (q, decode.run arguments,
    run keywords, plan tables (old_indptr, old_indices, exact_indptr,
    exact_indices, exact_last_page_len)).  page_gauge: the benchmark's
    gauge cache (INT8 pages + the 256-token exact ring); affine_group16:
    every completed page quantised by the bulk affine quantiser, the last
    16 pages read as FP16 from the dense cache."""
    import numpy as np
    import torch

    from .cache import build_gauge_cache, synthetic_dense_cache
    from .decode import split_tables
    from .quantize import quantize_pages

    q, dk, dv = synthetic_dense_cache(lengths, hkv=kv_heads, seed=seed, device="cuda")
    if representation == "page_gauge":
        c, t = build_gauge_cache(dk, dv, lengths)
        del dk, dv
        args = (c.key_codes, c.value_codes, c.key_scales, c.value_scales, c.exact_key,
                c.exact_value, c.value_center)
        return q, args, {}, (t.old_indptr, t.old_indices, t.exact_indptr, t.exact_indices,
                             t.exact_last_page_len)
    kc, kb, ks, _ = quantize_pages(dk)
    vc, vb, vs, _ = quantize_pages(dv)
    o_ptr, o_idx, e_ptr, e_idx = split_tables([-(-n // PAGE) for n in lengths], 16)
    last = torch.tensor([(n - 1) % PAGE + 1 for n in lengths], dtype=torch.int32,
                        device="cuda")
    tables = (o_ptr, torch.from_numpy(np.ascontiguousarray(o_idx)).cuda(), e_ptr,
              torch.from_numpy(np.ascontiguousarray(e_idx)).cuda(), last)
    return q, (kc, vc, ks, vs, dk, dv, None), {"affine_bias": (kb, vb)}, tables


def _sweep_steady(batch, context, repeats, seeds, write, path, lengths, layers, kv_heads=8,
                  representation="page_gauge"):
    import torch

    from .decode import PageGaugeDecode

    lengths = list(lengths) if lengths is not None else [context] * batch
    batch, context = len(lengths), max(lengths)
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    chunk = 8 * layers
    setups = []  # per seed: (q, per-layer (run arguments, keywords), plan tables)
    for seed in seeds:
        caches = []
        for layer in range(layers):
            q, args, kw, tables = _layer_setup(lengths, seed + 7919 * layer, kv_heads,
                                               representation)
            caches.append((args, kw))
        setups.append((q, caches, tables))
    out = torch.empty_like(setups[0][0])
    o_ptr = setups[0][2][0]
    old_pages = max(int(o_ptr[r + 1] - o_ptr[r]) for r in range(len(lengths)))

    def measure(split: int) -> float:
        per_seed = []
        for q, caches, tables in setups:
            dec = PageGaugeDecode(ws)
            dec.plan(*tables, 4 * kv_heads, kv_heads, old_split_pages=split)

            def run(c):
                dec.run(q, *c[0], out=out, **c[1])

            with torch.cuda.stream(stream):
                for c in caches:
                    run(c)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(chunk):
                        run(caches[i % layers])
                for _ in range(3):
                    graph.replay()
                times = []
                for _ in range(repeats):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    graph.replay()
                    e.record()
                    e.synchronize()
                    times.append(s.elapsed_time(e) * 1e3 / chunk)
            torch.cuda.synchronize()
            del graph
            per_seed.append(statistics.median(times))
        return statistics.fmean(per_seed)

    p50 = {split: measure(split) for split in candidates(old_pages)}
    # Refine around the best fixed size even when the heuristic (0) wins.
    fixed = {k: v for k, v in p50.items() if k > 0}
    for split in refinements(min(fixed, key=fixed.get), p50) if fixed else []:
        p50[split] = measure(split)
    del setups
    if write:
        record(batch, context, p50, path=path, kv_heads=kv_heads, representation=representation,
               meta={"gpu": torch.cuda.get_device_name(), "repeats": repeats,
                     "seeds": list(seeds), "lengths": lengths, "layers": layers,
                     "kv_heads": kv_heads, "representation": representation,
                     "mode": (f"steady: CUDA graph of {chunk} back-to-back decode steps "
                              f"(split + merge) cycling {layers} caches; coarse num_splits "
                              f"candidates, then +-20 % around the winner")})
    return p50


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--sweep", action="store_true")
    parser.add_argument("--batch", type=int, nargs="*", default=[1])
    parser.add_argument("--context", type=int, nargs="*", default=[49152])
    parser.add_argument("--repeats", type=int, default=60)
    parser.add_argument("--ragged", type=int, default=0,
                        help="also sweep a ragged batch of this size (contexts U[4096, 32768])")
    parser.add_argument("--table", type=Path, default=TABLE_PATH)
    parser.add_argument("--mode", choices=("steady", "burst"), default="steady")
    parser.add_argument("--kv-heads", type=int, nargs="*", default=[8],
                        help="KV heads per GPU (8 / tensor-parallel or head-shard degree)")
    parser.add_argument("--representation", choices=REPRESENTATIONS, default="page_gauge")
    parser.add_argument("--reset", action="store_true", help="start from an empty table")
    args = parser.parse_args()
    if args.reset and args.sweep:
        args.table.write_text(json.dumps({"entries": {}}, indent=1) + "\n")
    if not args.sweep:
        print(json.dumps(load_table(args.table), indent=1))
        return
    for h in args.kv_heads:
        for b in args.batch:
            for c in args.context:
                print(b, c, h, json.dumps(sweep(b, c, args.repeats, path=args.table,
                                                mode=args.mode, kv_heads=h,
                                                representation=args.representation)),
                      flush=True)
        if args.ragged:
            from .shard import ragged_lengths
            lengths = ragged_lengths(args.ragged, 20261001)
            print("ragged", lengths, h, json.dumps(sweep(0, 0, args.repeats, path=args.table,
                                                         lengths=lengths, mode=args.mode,
                                                         kv_heads=h,
                                                         representation=args.representation)),
                  flush=True)


if __name__ == "__main__":
    main()
