#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the reference itself.

Run once in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/PageGauge

It imports the reference's CPU-runnable Python (its PyTorch quantiser, its
page-table helpers) and evaluates the torch expressions its tests pin, on
seeded CPU tensors, and writes small .npz/.json fixtures.  The fixtures are
committed; tests never read the reference at run time.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load(ref: Path, name: str, rel: str):
    spec = importlib.util.spec_from_file_location(name, ref / rel)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def rope_tables(positions: int, theta: float = 1.0e6, dim: int = 128):
    """HF Mistral rotary tables: fp32 inv_freq, cat(freqs, freqs), cast fp16."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    t = torch.arange(positions, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().half(), emb.sin().half()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    ref = args.reference.resolve()
    affine = load(ref, "ref_affine", "scripts/benchmark_flashinfer_page_affine_int8.py")
    transformer = load(ref, "ref_transformer", "scripts/benchmark_page_gauge_transformer.py")

    # 1. quantize_page_gauge (scripts/benchmark_flashinfer_page_affine_int8.py:256-278)
    g = torch.Generator().manual_seed(20261001)
    mu = torch.randn(8, 128, generator=g) * math.sqrt(2.0)
    values = (torch.randn(3, 16, 8, 128, generator=g) + mu).half()
    codes, center, scale, recon, centered = affine.quantize_page_gauge(values)
    np.savez_compressed(
        HERE / "quantize_page_gauge.npz",
        values=values.numpy(), codes=codes.numpy(), center=center.numpy(),
        scale=scale.numpy(), reconstructed=recon.numpy(), centered=centered.numpy(),
    )

    # 2. RoPE pin (tests/test_page_gauge_append_extension.py:75-92): the torch
    # FP16 expression q*cos + cat(-q[64:], q[:64])*sin on CPU half tensors.
    g = torch.Generator().manual_seed(20261002)
    cos, sin = rope_tables(64)
    q = torch.randn(2, 32, 128, generator=g).half()
    k = (torch.randn(2, 8, 128, generator=g) * 2.0).half()
    positions = [0, 1, 15, 16, 37, 63]
    eq, ek = [], []
    for p in positions:
        c, s = cos[p], sin[p]
        eq.append(q * c + torch.cat((-q[..., 64:], q[..., :64]), dim=-1) * s)
        ek.append(k * c + torch.cat((-k[..., 64:], k[..., :64]), dim=-1) * s)
    np.savez_compressed(
        HERE / "rope.npz", q=q.numpy(), k=k.numpy(), cos=cos.numpy(), sin=sin.numpy(),
        positions=np.array(positions), expected_q=torch.stack(eq).numpy(),
        expected_k=torch.stack(ek).numpy(),
    )

    # 3. Completed-page scale algebra pin (tests/test_page_gauge_overheads.py:54-63).
    g = torch.Generator().manual_seed(21)
    key = torch.randn(3, 16, 2, 128, generator=g).half()
    kc = (torch.randn(2, 128, generator=g) * 0.1).half()
    expected = ((key.float() - kc[None, None].float()).permute(0, 2, 1, 3).abs()
                .amax(dim=(2, 3)).div(127.0).clamp_min(2.0**-20).half())
    np.savez_compressed(HERE / "scale_pin.npz", key=key.numpy(), center=kc.numpy(),
                        expected_scale=expected.numpy())

    # 4. Exact-tail merge oracle (tests/test_page_gauge_append_extension.py:588-676),
    # evaluated on CPU with the reference test's own einsum formula.
    g = torch.Generator().manual_seed(97)
    hq, hkv, dim, ring = 32, 8, 128, 16
    sm_scale = dim ** -0.5
    log2e = 1.4426950408889634
    query = torch.randn(1, hq, dim, generator=g).half()
    ek = (torch.randn(ring, 16, hkv, dim, generator=g) * 0.35).half()
    ev = (torch.randn(ring, 16, hkv, dim, generator=g) * 0.35).half()
    vc = (torch.randn(hkv, dim, generator=g) * 0.1).half()
    cases = {}
    for tail_tokens in (1, 15, 16, 17, 241, 255, 256):
        n = (tail_tokens + 15) // 16
        idx = torch.arange(7, 7 + n, dtype=torch.int32).remainder(ring)
        last = torch.tensor([(tail_tokens - 1) % 16 + 1], dtype=torch.int32)
        old_out = (torch.randn(1, hq, dim, generator=g) * 0.2).half()
        old_lse = torch.randn(1, hq, generator=g) * 0.5 + 8.0
        lk = ek[idx.long()].reshape(-1, hkv, dim)[:tail_tokens].float()
        lv = ev[idx.long()].reshape(-1, hkv, dim)[:tail_tokens].float()
        kvq = torch.arange(hq) // (hq // hkv)
        s = torch.einsum("qd,qtd->qt", query[0].float(), lk[:, kvq].permute(1, 0, 2)) * (sm_scale * log2e)
        mm = torch.maximum(old_lse[0], s.amax(dim=1))
        ow = torch.exp2(old_lse[0] - mm)
        tw = torch.exp2(s - mm[:, None])
        den = ow + tw.sum(dim=1)
        out = (ow[:, None] * old_out[0].float()
               + torch.einsum("qt,qtd->qd", tw, lv[:, kvq].permute(1, 0, 2))) / den[:, None]
        out = out + vc[kvq].float()
        cases[str(tail_tokens)] = dict(indices=idx.numpy(), last_len=last.numpy(),
                                       old_out=old_out.numpy(), old_lse=old_lse.numpy(),
                                       expected_out=out[None].numpy(),
                                       expected_lse=(torch.log2(den) + mm)[None].numpy())
    flat = {"query": query.numpy(), "exact_k": ek.numpy(), "exact_v": ev.numpy(),
            "value_center": vc.numpy()}
    for t, d in cases.items():
        for key_name, arr in d.items():
            flat[f"t{t}_{key_name}"] = arr
    np.savez_compressed(HERE / "tail_merge.npz", **flat)

    # 6. affine_group16 quantize_pages (scripts/benchmark_flashinfer_page_affine_int8.py:234-253):
    # random pages, a constant page (scale floor) and a page of exact
    # half-step ties (round half to even).
    g = torch.Generator().manual_seed(20261003)
    values = torch.randn(4, 16, 8, 128, generator=g) * 0.35
    values[1] = 0.75
    ramp = torch.arange(16 * 128, dtype=torch.float32).remainder(256).reshape(16, 128) * 0.125
    values[2] = ramp[:, None, :] + 0.0625  # (x - min) / (1/8) lands on k + 0.5
    values[2, 0, :, :] = 0.0
    values[2, 1, :, :] = 255 * 0.125
    values = values.half()
    a_codes, a_bias, a_scale, a_recon = affine.quantize_pages(values)
    np.savez_compressed(HERE / "quantize_affine_group16.npz", values=values.numpy(),
                        codes=a_codes.numpy(), bias=a_bias.numpy(), scale=a_scale.numpy(),
                        reconstructed=a_recon.numpy())

    # 5. Page-table helpers (scripts/benchmark_page_gauge_transformer.py:383-667;
    # scripts/benchmark_flashinfer_page_affine_int8.py:392-420).
    tables = {"segment_page_table": [], "request_major_page_table": [],
              "request_major_exact_page_table": [], "page_gauge_logical_partition": []}
    orig_tensor = torch.tensor

    def cpu_tensor(*a, **kw):
        kw["device"] = "cpu"
        return orig_tensor(*a, **kw)

    affine.torch.tensor = cpu_tensor  # segment_page_table allocates on "cuda"
    try:
        for rows, tail, sink in (([8, 6], 2, 1), ([20, 17, 33], 16, 0), ([5, 40], 4, 3)):
            outs = affine.segment_page_table(rows, tail, sink)
            tables["segment_page_table"].append(
                {"args": [rows, tail, sink], "out": [o.tolist() for o in outs]})
    finally:
        affine.torch.tensor = orig_tensor
    for args_ in ((2, 4, None), (2, 4, 2), (3, 7, 3)):
        out = transformer.request_major_page_table(args_[0], args_[1], args_[2], device="cpu")
        tables["request_major_page_table"].append({"args": list(args_), "out": out.tolist()})
    for args_ in ((2, 8, 2, 1), (2, 8, 2, 3), (3, 40, 16, 0), (1, 64, 16, 4)):
        out = transformer.request_major_exact_page_table(*args_, device="cpu")
        tables["request_major_exact_page_table"].append({"args": list(args_), "out": out.tolist()})
    for args_ in ((1283, 16, 1, 7), (8, 2, 3, 16), (3072, 16, 0, 16), (257, 16, 0, 1)):
        part = transformer.page_gauge_logical_partition(*args_)
        tables["page_gauge_logical_partition"].append({
            "args": list(args_),
            "out": {k: (list(v) if isinstance(v, tuple) else v) for k, v in part.items()},
        })
    (HERE / "page_tables.json").write_text(json.dumps(tables, indent=1) + "\n")
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
