"""GPU parity of the fused RoPE/append/finalise kernels and the bulk
quantiser.  Integer and FP16 storage outputs are compared bit-exactly with
the CPU oracle; scenarios follow tests/test_page_gauge_append_extension.py."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import pagegauge_oracle as O
from pagegauge_b200.cache import rope_tables
from pagegauge_b200.quantize import quantize_completed_kv_pages, quantize_page_gauge, quantize_pages_into
from pagegauge_b200.runtime import load_append_extension, read_device_error

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def u16(x):
    return np.asarray(x).view(np.uint16)


def cpu(t):
    return t.detach().cpu().numpy()


def _gauge_buffers(batch, exact_ppr, code_ppr, hkv=8):
    z = dict(device="cuda")
    return dict(
        exact_k=torch.zeros(batch * exact_ppr, 16, hkv, 128, dtype=torch.float16, **z),
        exact_v=torch.zeros(batch * exact_ppr, 16, hkv, 128, dtype=torch.float16, **z),
        codes_k=torch.zeros(batch * code_ppr, 16, hkv, 128, dtype=torch.int8, **z),
        codes_v=torch.zeros(batch * code_ppr, 16, hkv, 128, dtype=torch.int8, **z),
        scales_k=torch.zeros(batch * code_ppr, hkv, dtype=torch.float16, **z),
        scales_v=torch.zeros(batch * code_ppr, hkv, dtype=torch.float16, **z),
    )


def _oracle_state(batch, exact_ppr, code_ppr, hkv=8):
    return O.GaugeState(
        exact_k=np.zeros((batch * exact_ppr, 16, hkv, 128), np.float16),
        exact_v=np.zeros((batch * exact_ppr, 16, hkv, 128), np.float16),
        codes_k=np.zeros((batch * code_ppr, 16, hkv, 128), np.int8),
        codes_v=np.zeros((batch * code_ppr, 16, hkv, 128), np.int8),
        scales_k=np.zeros((batch * code_ppr, hkv), np.float16),
        scales_v=np.zeros((batch * code_ppr, hkv), np.float16),
    )


def _assert_state_equal(buf, st):
    assert np.array_equal(u16(cpu(buf["exact_k"])), u16(st.exact_k))
    assert np.array_equal(u16(cpu(buf["exact_v"])), u16(st.exact_v))
    assert np.array_equal(cpu(buf["codes_k"]), st.codes_k)
    assert np.array_equal(cpu(buf["codes_v"]), st.codes_v)
    assert np.array_equal(u16(cpu(buf["scales_k"])), u16(st.scales_k))
    assert np.array_equal(u16(cpu(buf["scales_v"])), u16(st.scales_v))


@pytest.mark.parametrize("batch,logical_pages,prefix,tail,shared_center", [
    (1, 4, 0, 2, True),     # ring reuse (reference :218-279)
    (1, 5, 1, 2, True),     # sink slot survives wraps (:282-349)
    (2, 8, 3, 2, False),    # S3 prefix, batched centres (:352-518)
    (3, 3, 0, 2, False),    # request-major batch (:679-829)
])
def test_append_page_gauge_bit_exact_vs_oracle(cuda_lib, batch, logical_pages, prefix, tail, shared_center):
    g = torch.Generator().manual_seed(20261003 + batch)
    positions = logical_pages * 16
    cos, sin = rope_tables(positions)
    q = torch.randn(batch, 32, 128, generator=g).half()
    keys = (torch.randn(positions, batch, 8, 128, generator=g) * 2.0).half()
    values = torch.randn(positions, batch, 8, 128, generator=g).half()
    cshape = (8, 128) if shared_center else (batch, 8, 128)
    kc = (torch.randn(*cshape, generator=g) * 0.5).half()
    vc = (torch.randn(*cshape, generator=g) * 0.1).half()
    ext = load_append_extension()
    buf_s = _gauge_buffers(batch, prefix + tail, logical_pages)
    buf_d = _gauge_buffers(batch, prefix + tail, logical_pages)
    st = _oracle_state(batch, prefix + tail, logical_pages)
    dq, dk, dv = q.cuda(), keys.cuda(), values.cuda()
    dcos, dsin, dkc, dvc = cos.cuda(), sin.cuda(), kc.cuda(), vc.cuda()
    rq_s = torch.empty_like(dq)
    rq_d = torch.empty_like(dq)
    pos_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    for p in range(positions):
        ext.rope_append_page_gauge(dq, dk[p], dv[p], dcos[p], dsin[p], dkc, dvc, rq_s,
                                   buf_s["exact_k"], buf_s["exact_v"], buf_s["codes_k"], buf_s["codes_v"],
                                   buf_s["scales_k"], buf_s["scales_v"], prefix, p)
        pos_dev.fill_(p)
        ext.rope_append_page_gauge_dynamic(dq, dk[p], dv[p], dcos, dsin, pos_dev, dkc, dvc, rq_d,
                                           buf_d["exact_k"], buf_d["exact_v"], buf_d["codes_k"],
                                           buf_d["codes_v"], buf_d["scales_k"], buf_d["scales_v"], prefix)
        rq = O.rope_append_page_gauge(st, q.numpy(), keys[p].numpy(), values[p].numpy(), cos[p].numpy(),
                                      sin[p].numpy(), kc.numpy(), vc.numpy(), prefix, p)
    torch.cuda.synchronize()
    assert read_device_error() == 0
    assert np.array_equal(u16(cpu(rq_s)), u16(rq))
    assert np.array_equal(u16(cpu(rq_d)), u16(rq))
    _assert_state_equal(buf_s, st)
    _assert_state_equal(buf_d, st)
    # Reconstruction quality gate of the reference tests (< 2 % relative).
    kcf = kc.float().reshape(-1 if shared_center else batch, 8, 128)
    recon = buf_s["codes_k"].float().cpu() * buf_s["scales_k"].float().cpu()[:, None, :, None]
    rot = O.rope_fp16(keys.numpy(), cos.numpy()[:, None, None, :], sin.numpy()[:, None, None, :])
    ref = torch.from_numpy(rot.astype(np.float32)).permute(1, 0, 2, 3).reshape(batch * logical_pages, 16, 8, 128)
    cen = kcf[None] if shared_center else kcf.repeat_interleave(logical_pages, 0)
    rel = ((recon + cen.reshape(-1, 1, 8, 128) - ref).norm() / ref.norm()).item()
    assert rel < 0.02


@pytest.mark.parametrize("shared_center", [False, True])
def test_batched_positions_bit_exact_vs_oracle(cuda_lib, shared_center):
    """Per-request positions (ragged serving batch): requests start at
    staggered in-page phases, so every step closes pages for some requests
    only (the append benchmark's mixed close pattern)."""
    batch = 1 if shared_center else 8
    exact_ppr, code_ppr, steps = 3, 8, 40
    g = torch.Generator().manual_seed(20261011 + batch)
    cos, sin = rope_tables(code_ppr * 16)
    q = torch.randn(steps, batch, 32, 128, generator=g).half()
    keys = (torch.randn(steps, batch, 8, 128, generator=g) * 2.0).half()
    values = torch.randn(steps, batch, 8, 128, generator=g).half()
    cshape = (8, 128) if shared_center else (batch, 8, 128)
    kc = (torch.randn(*cshape, generator=g) * 0.5).half()
    vc = (torch.randn(*cshape, generator=g) * 0.1).half()
    start = np.array([(r * 16) // batch + 7 * r for r in range(batch)], np.int32)
    ext = load_append_extension()
    buf = _gauge_buffers(batch, exact_ppr, code_ppr)
    f16k = torch.zeros(batch * code_ppr, 16, 8, 128, dtype=torch.float16, device="cuda")
    f16v = torch.zeros_like(f16k)
    st = _oracle_state(batch, exact_ppr, code_ppr)
    ok = np.zeros((batch * code_ppr, 16, 8, 128), np.float16)
    ov = np.zeros_like(ok)
    dcos, dsin, dkc, dvc = cos.cuda(), sin.cuda(), kc.cuda(), vc.cuda()
    rq = torch.empty(batch, 32, 128, dtype=torch.float16, device="cuda")
    rq16 = torch.empty_like(rq)
    pos_dev = torch.empty(batch, dtype=torch.int32, device="cuda")
    closes = 0
    for step in range(steps):
        pos = start + step
        closes += int((pos % 16 == 15).sum())
        pos_dev.copy_(torch.from_numpy(pos))
        dq, dk, dv = q[step].cuda(), keys[step].cuda(), values[step].cuda()
        ext.rope_append_page_gauge_batched(dq, dk, dv, dcos, dsin, pos_dev, dkc, dvc, rq,
                                           buf["exact_k"], buf["exact_v"], buf["codes_k"],
                                           buf["codes_v"], buf["scales_k"], buf["scales_v"], 0)
        ext.rope_append_fp16_batched(dq, dk, dv, dcos, dsin, pos_dev, rq16, f16k, f16v)
        orq = O.rope_append_page_gauge_batched(st, q[step].numpy(), keys[step].numpy(),
                                               values[step].numpy(), cos.numpy(), sin.numpy(),
                                               kc.numpy(), vc.numpy(), 0, pos)
        orq16 = O.rope_append_fp16_batched(ok, ov, q[step].numpy(), keys[step].numpy(),
                                           values[step].numpy(), cos.numpy(), sin.numpy(), pos)
        torch.cuda.synchronize()
        assert np.array_equal(u16(cpu(rq)), u16(orq))
        assert np.array_equal(u16(cpu(rq16)), u16(orq16))
    assert closes >= 2 * batch
    assert read_device_error() == 0
    _assert_state_equal(buf, st)
    assert np.array_equal(u16(cpu(f16k)), u16(ok))
    assert np.array_equal(u16(cpu(f16v)), u16(ov))


def test_batched_position_out_of_range_skips_only_that_request(cuda_lib):
    ext = load_append_extension()
    batch, exact_ppr, code_ppr = 4, 2, 4
    cos, sin = rope_tables(code_ppr * 16)
    g = torch.Generator().manual_seed(7)
    q = torch.randn(batch, 32, 128, generator=g).half().cuda()
    k = torch.randn(batch, 8, 128, generator=g).half().cuda()
    v = torch.randn(batch, 8, 128, generator=g).half().cuda()
    kc = torch.zeros(batch, 8, 128, dtype=torch.float16, device="cuda")
    buf = _gauge_buffers(batch, exact_ppr, code_ppr)
    rq = torch.zeros_like(q)
    pos = torch.tensor([3, code_ppr * 16, 5, -1], dtype=torch.int32, device="cuda")
    read_device_error()
    ext.rope_append_page_gauge_batched(q, k, v, cos.cuda(), sin.cuda(), pos, kc, kc, rq,
                                       buf["exact_k"], buf["exact_v"], buf["codes_k"],
                                       buf["codes_v"], buf["scales_k"], buf["scales_v"], 0)
    torch.cuda.synchronize()
    assert read_device_error() == 2  # kDevBadPosition
    ring = buf["exact_k"].view(batch, exact_ppr, 16, 8, 128)
    assert ring[0, 0, 3].abs().sum() > 0 and ring[2, 0, 5].abs().sum() > 0
    assert ring[1].abs().sum() == 0 and ring[3].abs().sum() == 0
    assert rq[1].abs().sum() == 0 and rq[3].abs().sum() == 0
    with pytest.raises(RuntimeError, match="one int32 per request"):
        ext.rope_append_page_gauge_batched(q, k, v, cos.cuda(), sin.cuda(), pos[:2], kc, kc, rq,
                                           buf["exact_k"], buf["exact_v"], buf["codes_k"],
                                           buf["codes_v"], buf["scales_k"], buf["scales_v"], 0)


def test_page_close_exact_ties_bit_exact(cuda_lib):
    """Centred values on exact code ties (x / scale = k + 0.5): page abs-max
    127/16 gives scale 1/16 exactly and values are multiples of 1/32, so
    half of them sit on a tie and the page close must round them as the
    IEEE quotient does (half away from zero)."""
    batch, exact_ppr, code_ppr = 2, 2, 2
    n = code_ppr * 16
    g = torch.Generator().manual_seed(99)
    cos = torch.ones(n, 128, dtype=torch.float16)
    sin = torch.zeros(n, 128, dtype=torch.float16)
    keys = (torch.randint(-254, 255, (n, batch, 8, 128), generator=g).float() / 32).half()
    values = (torch.randint(-254, 255, (n, batch, 8, 128), generator=g).float() / 32).half()
    for t in range(0, n, 16):
        keys[t, :, :, 0] = 127 / 16
        values[t, :, :, 1] = -127 / 16
    q = torch.randn(batch, 32, 128, generator=g).half()
    zero = torch.zeros(batch, 8, 128, dtype=torch.float16)
    ext = load_append_extension()
    buf = _gauge_buffers(batch, exact_ppr, code_ppr)
    st = _oracle_state(batch, exact_ppr, code_ppr)
    dq, dz, rq = q.cuda(), zero.cuda(), torch.empty(batch, 32, 128, dtype=torch.float16, device="cuda")
    for p in range(n):
        ext.rope_append_page_gauge(dq, keys[p].cuda(), values[p].cuda(), cos[p].cuda(), sin[p].cuda(),
                                   dz, dz, rq, buf["exact_k"], buf["exact_v"], buf["codes_k"],
                                   buf["codes_v"], buf["scales_k"], buf["scales_v"], 0, p)
        O.rope_append_page_gauge(st, q.numpy(), keys[p].numpy(), values[p].numpy(), cos[p].numpy(),
                                 sin[p].numpy(), zero.numpy(), zero.numpy(), 0, p)
    torch.cuda.synchronize()
    assert np.all(u16(st.scales_k) == u16(np.float16(1 / 16)))
    ties = (np.abs(st.exact_k.astype(np.float32) * 16) % 1 == 0.5).sum()
    assert ties > 1000
    _assert_state_equal(buf, st)


def test_rope_matches_golden_torch_expression(cuda_lib):
    """RoPE of the append kernel equals the reference's torch FP16 pin."""
    g = np.load(GOLDEN / "rope.npz")
    ext = load_append_extension()
    q = torch.from_numpy(g["q"]).cuda()
    k = torch.from_numpy(g["k"]).cuda()
    v = torch.zeros_like(k)
    cos, sin = torch.from_numpy(g["cos"]).cuda(), torch.from_numpy(g["sin"]).cuda()
    for i, p in enumerate(g["positions"]):
        rq = torch.empty_like(q)
        pages = torch.zeros(2 * 4, 16, 8, 128, dtype=torch.float16, device="cuda")
        vpages = torch.zeros_like(pages)
        ext.rope_append_fp16(q, k, v, cos[p], sin[p], rq, pages, vpages, int(p))
        torch.cuda.synchronize()
        assert np.array_equal(u16(cpu(rq)), u16(g["expected_q"][i]))
        for r in range(2):
            got = pages[r * 4 + int(p) // 16, int(p) % 16]
            assert np.array_equal(u16(cpu(got)), u16(g["expected_k"][i][r]))


def test_fp16_append_static_dynamic_and_oracle(cuda_lib):
    """tests/test_page_gauge_append_extension.py:21-92 on the FP16 path."""
    g = torch.Generator().manual_seed(20261003)
    batch, ppr = 2, 3
    cos = torch.randn(48, 128, generator=g).half()
    sin = torch.randn(48, 128, generator=g).half()
    q = torch.randn(batch, 32, 128, generator=g).half()
    keys = torch.randn(48, batch, 8, 128, generator=g).half()
    values = torch.randn(48, batch, 8, 128, generator=g).half()
    ext = load_append_extension()
    ks = torch.zeros(batch * ppr, 16, 8, 128, dtype=torch.float16, device="cuda")
    vs, kd, vd = torch.zeros_like(ks), torch.zeros_like(ks), torch.zeros_like(ks)
    rqs, rqd = torch.empty(batch, 32, 128, dtype=torch.float16, device="cuda"), \
        torch.empty(batch, 32, 128, dtype=torch.float16, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    okp = np.zeros((batch * ppr, 16, 8, 128), np.float16)
    ovp = np.zeros_like(okp)
    dq, dk, dv, dc, ds = q.cuda(), keys.cuda(), values.cuda(), cos.cuda(), sin.cuda()
    for p in range(48):
        ext.rope_append_fp16(dq, dk[p], dv[p], dc[p], ds[p], rqs, ks, vs, p)
        pos.fill_(p)
        ext.rope_append_fp16_dynamic(dq, dk[p], dv[p], dc, ds, pos, rqd, kd, vd)
        orq = O.rope_append_fp16(okp, ovp, q.numpy(), keys[p].numpy(), values[p].numpy(),
                                 cos[p].numpy(), sin[p].numpy(), p)
    torch.cuda.synchronize()
    assert torch.equal(ks, kd) and torch.equal(vs, vd) and torch.equal(rqs, rqd)
    assert np.array_equal(u16(cpu(ks)), u16(okp)) and np.array_equal(u16(cpu(vs)), u16(ovp))
    assert np.array_equal(u16(cpu(rqs)), u16(orq))


def test_append_validation_messages(cuda_lib):
    """Error strings of tests/test_page_gauge_append_extension.py:520-585."""
    ext = load_append_extension()
    b = 2
    q = torch.randn(b, 32, 128, device="cuda").half()
    k = torch.randn(b, 8, 128, device="cuda").half()
    cos = torch.ones(4, 128, device="cuda").half()
    sin = torch.zeros_like(cos)
    kc = torch.zeros(b, 8, 128, device="cuda").half()
    buf = _gauge_buffers(b, 5, 8)
    rq = torch.empty_like(q)
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = (buf["exact_k"], buf["exact_v"], buf["codes_k"], buf["codes_v"], buf["scales_k"], buf["scales_v"])
    with pytest.raises(RuntimeError, match="must be nonnegative"):
        ext.rope_append_page_gauge(q, k, k, cos[0], sin[0], kc, kc, rq, *args, -1, 0)
    with pytest.raises(RuntimeError, match="at least one tail-ring page"):
        ext.rope_append_page_gauge_dynamic(q, k, k, cos, sin, pos, kc, kc, rq, *args, 5)
    big = _gauge_buffers(b, 10, 8)
    with pytest.raises(RuntimeError, match="logical cache capacity"):
        ext.rope_append_page_gauge(q, k, k, cos[0], sin[0], kc, kc, rq, big["exact_k"], big["exact_v"],
                                   buf["codes_k"], buf["codes_v"], buf["scales_k"], buf["scales_v"], 8, 0)
    with pytest.raises(RuntimeError, match="per-request PageGauge cache capacity"):
        ext.rope_append_page_gauge(q, k, k, cos[0], sin[0], kc, kc, rq, *args, 0, 8 * 16)
    with pytest.raises(RuntimeError, match="head-major"):
        ext.rope_append_page_gauge(q.transpose(1, 2).contiguous().transpose(1, 2), k, k, cos[0], sin[0],
                                   kc, kc, rq, *args, 0, 0)


def test_dynamic_position_out_of_range_is_skipped_and_flagged(cuda_lib):
    """A device position outside the RoPE table or cache writes nothing and
    raises the device guard word (no trap)."""
    ext = load_append_extension()
    q = torch.randn(1, 32, 128, device="cuda").half()
    k = torch.randn(1, 8, 128, device="cuda").half()
    cos = torch.ones(8, 128, device="cuda").half()
    buf = _gauge_buffers(1, 2, 4)
    rq = torch.zeros_like(q)
    pos = torch.full((1,), 100, dtype=torch.int32, device="cuda")
    read_device_error()
    ext.rope_append_page_gauge_dynamic(q, k, k, cos, cos, pos, k[0], k[0], rq, buf["exact_k"], buf["exact_v"],
                                       buf["codes_k"], buf["codes_v"], buf["scales_k"], buf["scales_v"], 0)
    torch.cuda.synchronize()
    assert read_device_error() == 2
    assert int(buf["exact_k"].abs().sum().item()) == 0 and int(rq.abs().sum().item()) == 0


def test_bulk_quantizer_matches_reference_quantize_page_gauge(cuda_lib):
    g = np.load(GOLDEN / "quantize_page_gauge.npz")
    values = torch.from_numpy(g["values"]).cuda()
    center = torch.from_numpy(g["center"]).cuda()
    codes = torch.empty_like(values, dtype=torch.int8)
    codes2 = torch.empty_like(codes)
    scales = torch.empty(values.shape[0], 8, dtype=torch.float16, device="cuda")
    scales2 = torch.empty_like(scales)
    quantize_pages_into(values, values, center, center, codes, codes2, scales, scales2, 0, "half_even")
    torch.cuda.synchronize()
    assert np.array_equal(cpu(codes), g["codes"])
    assert np.array_equal(u16(cpu(scales)), u16(g["scale"]))
    c2, center2, s2, recon, centered = quantize_page_gauge(values)
    torch.cuda.synchronize()
    assert np.abs(u16(cpu(center2)).astype(int) - u16(g["center"]).astype(int)).max() <= 1
    rel = ((recon.float() - centered.float()).norm() / centered.float().norm()).item()
    assert rel < 0.02


def test_completed_page_quantizer_scale_pin(cuda_lib):
    """tests/test_page_gauge_overheads.py:20-63 with the torch scale pin."""
    g = np.load(GOLDEN / "scale_pin.npz")
    key = torch.from_numpy(g["key"]).cuda()
    kc = torch.from_numpy(g["center"]).cuda()
    codes = torch.empty_like(key, dtype=torch.int8)
    scales = torch.empty(3, 2, dtype=torch.float16, device="cuda")
    quantize_completed_kv_pages(key, key, kc, kc, codes, torch.empty_like(codes), scales,
                                torch.empty_like(scales))
    torch.cuda.synchronize()
    assert np.array_equal(u16(cpu(scales)), u16(g["expected_scale"]))
    oc, os_ = O.quantize_pages_bulk(g["key"], g["center"], "half_away")
    assert np.array_equal(cpu(codes), oc)
    recon = codes.float() * scales[:, None, :, None].float() + kc[None, None].float()
    assert ((recon - key.float()).norm() / key.float().norm()).item() < 0.02
