"""Query distributions beyond N(0,1) for the INT8 QK path, and a CPU model
of the kernel's int8 query decomposition.

The INT8 segment multiplies the query by the K codes on the integer tensor
path, so each FP16 query row is first written as int8 parts sharing one
scale per row, sq = max|q_row| / 127:

    q ~ sq * (hi + lo/254 + lo2/254^2)

(``pg_decode_int8.cuh``, ``load_q_int8``).  The reference multiplies the
FP16 query by the exactly converted codes instead
(patches/flashinfer-0.6.17-page-gauge-int8.patch:61-77), so the
decomposition's error is the one place where the INT8 path's arithmetic
departs from the reference's.  It scales with the row's largest channel,
which is why the rows below carry outlier channels."""

from __future__ import annotations

import numpy as np
import torch

from pagegauge_b200.cache import apply_rope_fp16, rope_tables

KINDS = ("x20", "x100", "x300", "dominant", "rope")


def outlier_queries(batch: int, hq: int, kind: str, seed: int, position: int = 4095) -> torch.Tensor:
    """FP16 queries [batch, hq, 128] on the CPU.

    ``xF``: N(0,1) rows with 4 random channels per head scaled by F;
    ``dominant``: 0.01*N(0,1) rows with one channel per head set to 60;
    ``rope``: per-(head, channel) scales exp(1.2*N(0,1)) (three decades,
    the spread of real post-RoPE queries) rotated by RoPE at ``position``."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, hq, 128, generator=g)
    if kind.startswith("x"):
        f = float(kind[1:])
        for h in range(hq):
            ch = torch.randperm(128, generator=g)[:4]
            q[:, h, ch] *= f
    elif kind == "dominant":
        q *= 0.01
        for h in range(hq):
            c = int(torch.randint(0, 128, (1,), generator=g))
            q[:, h, c] = 60.0
    elif kind == "rope":
        scale = torch.exp(torch.randn(hq, 128, generator=g) * 1.2)
        x = (q * scale).half()
        cos, sin = rope_tables(position + 1)
        return torch.stack([apply_rope_fp16(x[b:b + 1], cos[position:position + 1],
                                            sin[position:position + 1])[0]
                            for b in range(batch)])
    else:
        raise ValueError(kind)
    return q.half()


def split_query(q: np.ndarray, parts: int) -> np.ndarray:
    """The value the kernel's int8 query parts represent (float64), for
    rows of the last axis: FP32 arithmetic as in ``load_q_int8``."""
    q = np.asarray(q, np.float32)
    amax = np.abs(q).max(-1, keepdims=True)
    sq = np.where(amax > 0, amax / np.float32(127), np.float32(1)).astype(np.float32)
    hi = np.clip(np.rint(q * (np.float32(1) / sq)), -127, 127).astype(np.float32)
    rem = (q - hi * sq).astype(np.float32)
    lo = np.clip(np.rint(rem * (np.float32(254) / sq)), -127, 127).astype(np.float32)
    rec = hi.astype(np.float64) + lo / 254.0
    if parts == 3:
        rem2 = (rem - lo * (sq / np.float32(254))).astype(np.float32)
        lo2 = np.clip(np.rint(rem2 * (np.float32(64516) / sq)), -127, 127)
        rec = rec + lo2 / 64516.0
    return rec * sq.astype(np.float64)
