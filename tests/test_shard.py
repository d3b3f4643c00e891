"""Request sharding across ranks (B8 ragged, no data-path collective): the
host partition, its byte model, and a world-size-2 gloo run on CPU in which
each rank decodes its own requests (CPU oracle standing in for the GPU
kernels) and rank 0 gathers the outputs back into request order."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pagegauge_oracle as O
from pagegauge_b200.cache import synthetic_dense_cache
from pagegauge_b200.decode import split_tables
from pagegauge_b200.shard import (gather_outputs, ragged_lengths, request_bytes, shard_loads,
                                  shard_requests)


def _bench_bytes(lengths, tail_pages=16):
    """Bytes from the CSR split of the decode tables (old pages full)."""
    pages = [-(-n // 16) for n in lengths]
    o_ptr, _, _, _ = split_tables(pages, tail_pages)
    total = 0
    for r, n in enumerate(lengths):
        old = int(o_ptr[r + 1] - o_ptr[r])
        exact_tokens = n - 16 * old
        total += 2 * 16 * old * 8 * 128 + old * 8 * 4 + 2 * exact_tokens * 8 * 128 * 2
    return total


def test_ragged_lengths_prefix_is_the_b8_config():
    b8 = ragged_lengths(8, 20261001)
    assert all(4096 <= n <= 32768 for n in b8)
    assert ragged_lengths(32, 20261001)[:8] == b8  # weak scaling keeps the first 8 (B8 ragged)


@pytest.mark.parametrize("lengths", [[49152], [1, 15, 16, 17, 255, 256, 257, 4097],
                                     ragged_lengths(8, 20261001)])
def test_request_bytes_match_table_split(lengths):
    assert sum(request_bytes(n) for n in lengths) == _bench_bytes(lengths)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_partition_and_balance(world):
    lengths = ragged_lengths(8 * world, 20261002)
    shards = shard_requests(lengths, world)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lengths)))
    assert shards == shard_requests(lengths, world)  # deterministic
    loads = shard_loads(lengths, shards)
    biggest = max(request_bytes(n) for n in lengths)
    assert max(loads) - min(loads) <= biggest
    # Longest-first packing is within 4/3 of the ideal makespan.
    assert max(loads) <= 4 / 3 * max(sum(loads) / world, biggest) + 1


def test_more_ranks_than_requests_leaves_empty_shards():
    shards = shard_requests([5000, 300], 4)
    assert sorted(len(s) for s in shards) == [0, 0, 1, 1]


def _decode_requests(lengths, ids, seed):
    """CPU oracle decode of requests ``ids`` (each built from its own seed)."""
    outs = []
    for i in ids:
        n = lengths[i]
        q, dk, dv = synthetic_dense_cache([n], seed=seed + i)
        q, dk, dv = q.numpy(), dk.numpy(), dv.numpy()
        pages = -(-n // 16)
        tail = min(4, pages)
        ck_c = dk.reshape(-1, 8, 128)[:n].astype(np.float32).mean(0).astype(np.float16)
        cv_c = dv.reshape(-1, 8, 128)[:n].astype(np.float32).mean(0).astype(np.float16)
        ck, sk = O.quantize_pages_bulk(dk, ck_c)
        cv, sv = O.quantize_pages_bulk(dv, cv_c)
        ek = (dk[pages - tail:].astype(np.float32) - ck_c.astype(np.float32)).astype(np.float16)
        ev = (dv[pages - tail:].astype(np.float32) - cv_c.astype(np.float32)).astype(np.float16)
        old = list(range(pages - tail))
        out, _ = O.page_gauge_decode(q[0], ck, cv, sk, sv, old, 16 * len(old), ek, ev,
                                     list(range(tail)), n - 16 * len(old), cv_c, 128 ** -0.5)
        outs.append(out)
    return np.stack(outs) if outs else np.zeros((0, 32, 128))


def _rank_main(rank, world, port, lengths, seed, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = shard_requests(lengths, world)
        mine = _decode_requests(lengths, shards[rank], seed)
        gathered = [None] * world
        dist.all_gather_object(gathered, (shards[rank], mine))
        if rank == 0:
            idx = [g[0] for g in gathered]
            full = gather_outputs(idx, [g[1] for g in gathered], len(lengths))
            np.save(result_path, full)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_shard_and_gather_matches_single_process(tmp_path):
    lengths = [300, 1000, 40, 700, 513]
    seed = 4242
    path = str(tmp_path / "full.npy")
    mp.spawn(_rank_main, args=(2, _free_port(), lengths, seed, path), nprocs=2, join=True)
    full = np.load(path)
    ref = _decode_requests(lengths, list(range(len(lengths))), seed)
    assert full.shape == ref.shape
    assert np.array_equal(full, ref)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plan_shards_balances_bytes(world):
    from pagegauge_b200.shard import plan_shards, ragged_lengths, request_bytes

    for seed in (20261001, 20261002, 20261003):
        lengths = ragged_lengths(8, seed)
        total = sum(request_bytes(n) for n in lengths)
        plan = plan_shards(lengths, world)
        assert sum(plan["rank_bytes"]) == total or plan["mode"] == "heads"
        if plan["mode"] == "requests":
            assert max(plan["rank_bytes"]) <= total / world * 1.02
            assert sorted(sum(plan["requests"], [])) == list(range(8))
        else:
            # every rank: all requests over its own 8/world heads, 1/world of the bytes
            assert plan["heads"] == [(r * 8 // world, (r + 1) * 8 // world) for r in range(world)]
            assert all(req == list(range(8)) for req in plan["requests"])
            assert sum(plan["rank_bytes"]) == total
    # one long request among short ones on 8 GPUs: heads
    assert plan_shards([32768] + [4096] * 7, 8)["mode"] == "heads"
    assert plan_shards([4096] * 8, 8)["mode"] == "requests"


def test_head_shards_gather_to_the_whole_batch():
    from pagegauge_b200.shard import gather_head_outputs

    full = np.random.default_rng(0).standard_normal((8, 32, 128))
    parts = [full[:, 8 * r:8 * (r + 1)] for r in range(4)]  # 2 KV heads x group 4 each
    assert np.array_equal(gather_head_outputs(parts, 4), full)
