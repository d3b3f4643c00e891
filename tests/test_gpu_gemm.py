"""GPU parity of the weight-streaming skinny GEMM (decoder projections)
against a plain PyTorch FP32 reference of the same op, for the three
epilogues, stream-K splits that put several tiles in one CTA and several
CTAs on one tile, and batch sizes 1..32.  FP16 outputs may differ from the
FP32-then-FP16 reference by one FP16 rounding step (different summation
order); repeated runs must be bit-identical."""

from __future__ import annotations

import pytest
import torch

from pagegauge_b200.gemm import RESIDUAL, SILU_MUL, STORE, PackedWeight, SkinnyGemm
from pagegauge_b200.runtime import read_device_error

pytestmark = pytest.mark.gpu


def _data(n, k, batch, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).half()
    x = torch.randn(batch, k, generator=g, device="cuda").half()
    return w, x


def _ref(x, w):
    # Float64 on the device: no TF32 or reduced-precision path can enter.
    return (x.double() @ w.double().t()).float()


def _ulp16(x):
    """One FP16 unit in the last place at |x| (subnormal spacing below 2^-14)."""
    e = torch.floor(torch.log2(x.abs().float().clamp_min(2.0 ** -14)))
    return torch.exp2(e - 10)


def _assert_f16_close(got, ref, k):
    # One FP16 rounding step of the reference value, plus the FP32
    # accumulation error of a k-long dot product of these magnitudes
    # (~2^-24 * sqrt(k) * |partial sums|; 1e-6 * sqrt(k) leaves a wide margin).
    tol = ref.abs() * 2.0 ** -10 + 1e-6 * k ** 0.5
    err = (got.float() - ref).abs()
    assert bool((err <= tol).all()), f"max err {err.max().item():.3e}"


@pytest.mark.parametrize("n,k,batch,grid", [
    (256, 512, 1, 0), (6144, 4096, 1, 0), (4096, 4096, 5, 0), (1024, 14336, 32, 0),
    (512, 1024, 9, 7), (512, 1024, 16, 1), (4096, 4096, 32, 0), (768, 2048, 3, 50)])
def test_store_matches_torch(cuda_lib, n, k, batch, grid):
    w, x = _data(n, k, batch, n + k + batch)
    gemm = SkinnyGemm("cuda")
    gemm.reserve(n, k, batch)
    pw = PackedWeight(w)
    out = gemm(x, pw, grid=grid)
    again = gemm(x, pw, grid=grid)
    torch.cuda.synchronize()
    assert read_device_error() == 0
    _assert_f16_close(out, _ref(x, w), k)
    assert torch.equal(out, again)
    assert int(gemm.counters.abs().sum()) == 0


@pytest.mark.parametrize("batch", [1, 4, 32])
def test_residual_epilogue(cuda_lib, batch):
    """residual = f16(residual + f16(acc)): the residual mode splits the
    work exactly as the store mode does, so it must equal the store mode's
    output added to the residual, bit for bit."""
    n, k = 4096, 14336
    w, x = _data(n, k, batch, 11 + batch)
    g = torch.Generator(device="cuda").manual_seed(99 + batch)
    r0 = torch.randn(batch, n, generator=g, device="cuda").half()
    r = r0.clone()
    gemm = SkinnyGemm("cuda")
    gemm.reserve(n, k, batch, RESIDUAL)
    pw = PackedWeight(w)
    gemm(x, pw, mode=RESIDUAL, residual=r)
    y = gemm(x, pw)
    torch.cuda.synchronize()
    _assert_f16_close(y, _ref(x, w), k)
    assert torch.equal(r, r0 + y)


@pytest.mark.parametrize("batch,grid", [(1, 0), (8, 0), (32, 0), (5, 33)])
def test_silu_mul_epilogue(cuda_lib, batch, grid):
    f, k = 2048, 4096
    w, x = _data(2 * f, k, batch, 7 + batch)
    gemm = SkinnyGemm("cuda")
    gemm.reserve(2 * f, k, batch, SILU_MUL)
    out = gemm(x, PackedWeight(w, SILU_MUL), mode=SILU_MUL, grid=grid)
    torch.cuda.synchronize()
    acc = _ref(x, w)
    gate = acc[:, :f].half().float()
    up = acc[:, f:].half().float()
    s = (gate / (1 + torch.exp(-gate))).half().float()
    exp = (s * up).half()
    # gate and up may each move by one FP16 step (summation order), which
    # moves the product by about that relative amount, plus its rounding.
    diff = (out.float() - exp.float()).abs()
    # gate and up may each differ by one FP16 step or by the FP32
    # accumulation error e (absolute; it dominates near zero, where FP16
    # steps are tiny).  |d silu / dg| <= 1.1, so gate moves silu by at most
    # 1.1 * (ulp + e) and silu's own rounding by one more step, times |up|;
    # up moves the product by |silu(gate)| * (ulp + e).
    e = 1e-6 * k ** 0.5
    tol = (1.1 * (_ulp16(gate) + e) + _ulp16(s)) * up.abs() + s.abs() * (_ulp16(up) + e) \
        + _ulp16(exp)
    assert bool((diff <= tol).all()), (diff - tol).max().item()


def test_strided_operands_and_graph_replay(cuda_lib):
    n, k, batch = 1024, 2048, 3
    w, _ = _data(n, k, batch, 5)
    big = torch.randn(batch, k + 64, device="cuda").half()
    x = big[:, 32:32 + k]          # row stride k + 64, 64-byte offset
    out_big = torch.zeros(batch, n + 8, dtype=torch.float16, device="cuda")
    out = out_big[:, :n]
    gemm = SkinnyGemm("cuda")
    gemm.reserve(n, k, batch)
    pw = PackedWeight(w)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gemm(x, pw, out=out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            gemm(x, pw, out=out)
        out.zero_()
        graph.replay()
        graph.replay()
    torch.cuda.synchronize()
    _assert_f16_close(out, _ref(x, w), k)
    assert bool((out_big[:, n:] == 0).all())
    assert int(gemm.counters.abs().sum()) == 0


def test_rejects_bad_shapes(cuda_lib):
    gemm = SkinnyGemm("cuda")
    w, x = _data(256, 512, 2, 1)
    with pytest.raises(RuntimeError, match="multiples of 64"):
        PackedWeight(w[:, :500].contiguous())
    pw = PackedWeight(w)
    with pytest.raises(RuntimeError, match="batch must be 1..32"):
        gemm(torch.zeros(33, 512, dtype=torch.float16, device="cuda"), pw)
    with pytest.raises(ValueError, match="another epilogue"):
        gemm(x, pw, mode=SILU_MUL)


def test_packed_layout(cuda_lib):
    """Tile t, k-block kb, row r, 16-byte chunk c ^ (r & 7) holds
    W[64t + r, 64kb + 8c .. +8]; silu_mul tiles take 32 gate + 32 up rows."""
    n, k = 128, 192
    w = torch.arange(n * k, device="cuda").remainder(2039).half().view(n, k)
    for mode in (STORE, SILU_MUL):
        pw = PackedWeight(w, mode).data.view(-1, k // 64, 64, 8, 8)
        for t, kb, r, c in ((0, 0, 0, 0), (1, 2, 13, 5), (0, 1, 40, 7), (1, 0, 63, 3)):
            if mode == STORE:
                row = 64 * t + r
            else:
                row = 32 * t + r if r < 32 else n // 2 + 32 * t + (r - 32)
            assert torch.equal(pw[t, kb, r, c ^ (r & 7)], w[row, 64 * kb + 8 * c:64 * kb + 8 * c + 8])


def _rms_norm_ref(x, w, eps=1e-5):
    """transformers MistralRMSNorm on FP16 rows: f16(w * f16(x * rsqrt(ms + eps)))."""
    xf = x.float()
    inv = torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)
    return (w.float() * (xf * inv).half().float()).half()


@pytest.mark.parametrize("mode,batch,grid", [(STORE, 1, 0), (STORE, 5, 0), (SILU_MUL, 1, 0),
                                             (SILU_MUL, 8, 37), (STORE, 32, 0)])
def test_fused_rms_norm_prologue(cuda_lib, mode, batch, grid):
    """The GEMM's RMSNorm prologue equals normalising first and multiplying
    after: the normalised FP16 input may differ by one FP16 step where the
    two reductions round the mean square differently."""
    n, k = (2048, 4096) if mode == SILU_MUL else (1536, 4096)
    w, _ = _data(n, k, batch, 41 + batch)
    g = torch.Generator(device="cuda").manual_seed(7 * batch)
    x = (torch.randn(batch, k, generator=g, device="cuda") * 3).half()
    nw = (1 + 0.1 * torch.randn(k, generator=g, device="cuda")).half()
    gemm = SkinnyGemm("cuda")
    gemm.reserve(n, k, batch, mode)
    pw = PackedWeight(w, mode)
    fused = gemm(x, pw, mode=mode, grid=grid, norm_weight=nw)
    xn = _rms_norm_ref(x, nw)
    plain = gemm(xn, pw, mode=mode, grid=grid)
    torch.cuda.synchronize()
    assert read_device_error() == 0
    assert torch.equal(x, x)  # the input rows are read, never written
    if mode == STORE:
        ref = _ref(xn, w)
        slack = (xn.float().abs() * 2.0 ** -11) @ w.float().abs().t()
        tol = ref.abs() * 2.0 ** -10 + 1e-6 * k ** 0.5 + slack
        assert bool(((fused.float() - ref).abs() <= tol).all())
    # Against the two-step path: identical except for rare one-step input
    # differences.
    diff = (fused.float() - plain.float()).abs()
    assert diff.max().item() < 2e-2 and (diff == 0).float().mean().item() > 0.9
    with pytest.raises(ValueError, match="norm_weight"):
        gemm(x, pw, mode=mode, norm_weight=nw[:100])
