"""The decoder oracle pinned against transformers' MistralForCausalLM, the
product's tensor-parallel weight sharding checked on a world-size-2 gloo
run of the oracle, and the vocabulary-parallel greedy combine (CPU only)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import decoder_oracle as D
from pagegauge_b200.decoder import (DecoderConfig, TensorParallel, full_layer_tensors,
                                    full_model_tensors, pick_greedy, shard_layer)

TINY = DecoderConfig(layers=2, hidden=512, heads=4, kv_heads=2, intermediate=1024, vocab=256)
SEED = 31


def oracle_weights(cfg, tp=None, seed=SEED):
    tp = tp or TensorParallel.of(cfg)
    top = full_model_tensors(cfg, seed, "cpu")
    layers = []
    for l in range(cfg.layers):
        lw = shard_layer(cfg, tp, full_layer_tensors(cfg, seed, l, "cpu"))
        layers.append({k: getattr(lw, k).numpy() for k in
                       ("attn_norm", "qkv", "o", "mlp_norm", "gate_up", "down")})
    v0, v1 = tp.vocab
    return {"embed": top["embed"].numpy(), "final_norm": top["final_norm"].numpy(),
            "lm_head": top["lm_head"][v0:v1].numpy(), "layers": layers}


def oracle_cfg(cfg, tp=None):
    tp = tp or TensorParallel.of(cfg)
    return {"hq": tp.q_heads[1] - tp.q_heads[0], "hkv": tp.kv_heads[1] - tp.kv_heads[0],
            "eps": cfg.rms_eps, "theta": cfg.rope_theta}


def hf_model(cfg, seed=SEED):
    from transformers import MistralConfig, MistralForCausalLM

    hf = MistralForCausalLM(MistralConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
        num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim, rope_theta=cfg.rope_theta,
        rms_norm_eps=cfg.rms_eps, max_position_embeddings=1024, tie_word_embeddings=False)).eval()
    top = full_model_tensors(cfg, seed, "cpu")
    sd = {"model.embed_tokens.weight": top["embed"], "model.norm.weight": top["final_norm"],
          "lm_head.weight": top["lm_head"]}
    names = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
             "o": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj",
             "down": "mlp.down_proj", "attn_norm": "input_layernorm",
             "mlp_norm": "post_attention_layernorm"}
    for l in range(cfg.layers):
        for k, t in full_layer_tensors(cfg, seed, l, "cpu").items():
            sd[f"model.layers.{l}.{names[k]}.weight"] = t
    hf.load_state_dict({k: v.float() for k, v in sd.items()})
    return hf


def test_dense_oracle_matches_transformers_mistral():
    tokens = torch.randint(0, TINY.vocab, (40,), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        ref = hf_model(TINY)(tokens[None]).logits[0, -1].numpy()
    got, _ = D.dense_forward(oracle_weights(TINY), oracle_cfg(TINY), tokens.numpy(), round16=False)
    assert np.abs(got - ref).max() < 2e-5 * max(1.0, np.abs(ref).max())


def test_fp16_rounding_mode_stays_close_to_fp32():
    tokens = np.arange(0, 64, 3) % TINY.vocab
    w, c = oracle_weights(TINY), oracle_cfg(TINY)
    a, _ = D.dense_forward(w, c, tokens, round16=False)
    b, _ = D.dense_forward(w, c, tokens, round16=True)
    assert np.abs(a - b).max() < 5e-3
    assert np.dot(a, b) / np.linalg.norm(a) / np.linalg.norm(b) > 0.9999


def test_page_tables_window():
    tables = D.page_tables([0, 15, 16, 255, 256, 300], capacity_pages=40)
    assert tables[0] == ([], [0], 0, 1)
    assert tables[1] == ([], [16], 0, 16)
    assert tables[2] == ([], [32, 33], 0, 17)
    assert tables[3][0] == [] and len(tables[3][1]) == 16 and tables[3][3] == 256
    old, exact, ot, et = tables[4]
    assert old == [160] and exact == [64 + p % 16 for p in range(1, 17)] and (ot, et) == (16, 241)
    old, exact, ot, et = tables[5]
    assert old == [200 + p for p in range(3)] and ot == 48 and et == 253


def test_product_page_tables_match_oracle():
    from pagegauge_b200.decoder import page_tables

    pos = [0, 15, 16, 255, 256, 300, 1000]
    o_ptr, o_idx, e_ptr, e_idx = page_tables(pos, 70)
    for r, (old, exact, _, _) in enumerate(D.page_tables(pos, 70)):
        assert list(o_idx[o_ptr[r]:o_ptr[r + 1]]) == old
        assert list(e_idx[e_ptr[r]:e_ptr[r + 1]]) == exact


@pytest.mark.parametrize("sink,suffix,ring", [(1, 0, 4), (4, 0, 48), (1, 2, 4), (0, 3, 2)])
def test_product_page_tables_with_exact_policies_match_oracle(sink, suffix, ring):
    from pagegauge_b200.decoder import page_tables

    initial = 20
    pos = [initial * 16 + d for d in (0, 5, 16, 40, 77, 400)]
    o_ptr, o_idx, e_ptr, e_idx = page_tables(pos, 64, ring, sink, suffix, initial)
    for r, (old, exact, ot, et) in enumerate(D.page_tables(pos, 64, ring, sink, suffix, initial)):
        assert list(o_idx[o_ptr[r]:o_ptr[r + 1]]) == old
        assert list(e_idx[e_ptr[r]:e_ptr[r + 1]]) == exact
        # Exact-once cover of the context, current page last.
        assert ot + et == pos[r] + 1
        assert exact[-1] == r * (sink + suffix + ring) + sink + suffix + (pos[r] // 16) % ring


def test_pick_greedy_ties_and_order():
    # [world, B, (value, index)]; rank slices are ascending vocabulary ranges.
    pairs = torch.tensor([[[1.0, 3.0], [5.0, 1.0]],
                          [[2.0, 10.0], [5.0, 12.0]]])
    assert pick_greedy(pairs).tolist() == [10, 1]


def _tp_rank(rank, world, port, tokens, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tp = TensorParallel.of(TINY, rank, world)

        def reduce(x):
            t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        logits, _ = D.dense_forward(oracle_weights(TINY, tp), oracle_cfg(TINY, tp), tokens,
                                    reduce=reduce, round16=False)
        parts = [None] * world
        dist.all_gather_object(parts, logits)
        if rank == 0:
            np.save(result, np.concatenate(parts))
    finally:
        dist.destroy_process_group()


def test_two_rank_tensor_parallel_shards_reproduce_the_model(tmp_path):
    tokens = (np.arange(24) * 7) % TINY.vocab
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "tp.npy")
    mp.spawn(_tp_rank, args=(2, port, tokens, path), nprocs=2, join=True)
    full, _ = D.dense_forward(oracle_weights(TINY), oracle_cfg(TINY), tokens, round16=False)
    got = np.load(path)
    assert got.shape == full.shape
    assert np.abs(got - full).max() < 1e-5


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tensor_parallel_slices_cover_the_model(world):
    cfg = DecoderConfig()
    tps = [TensorParallel.of(cfg, r, world) for r in range(world)]
    for field in ("q_heads", "kv_heads", "intermediate", "vocab"):
        spans = [getattr(t, field) for t in tps]
        assert spans[0][0] == 0 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert tps[-1].q_heads[1] == 32 and tps[-1].kv_heads[1] == 8
    assert all((t.q_heads[1] - t.q_heads[0]) == 4 * (t.kv_heads[1] - t.kv_heads[0]) for t in tps)
    with pytest.raises(ValueError):
        TensorParallel.of(cfg, 0, 3)
