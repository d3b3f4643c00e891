// INT8 PageGauge pages of the split-KV decode (segment 0, one FP16 scale
// per (page, KV head)): Q split into three int8 parts for the integer MMA,
// QK on IMMA with the K scale applied to the fp32 scores, the V scale
// folded into P for an FP16 PV on biased codes, and the per-warp TMA
// pipeline that takes the pages two at a time.
#pragma once

#include "pg_decode_core.cuh"

namespace pg {

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | (static_cast<uint32_t>(d) << 24);
}

__device__ __forceinline__ int clamp127(int v) { return v < -127 ? -127 : (v > 127 ? 127 : v); }

// Three-part int8 Q for the INT8 segment, computed once per CTA into the
// shared table (all warps call this after the query is final, then read
// their fragments).  GQA <= 4: warp w splits query rows g = w, w + W, ...
// (< 4) and writes two of the eight mma lane-group slots, slot g with
// (hi, lo) and slot g + 4 with (lo2, 0), so each row is loaded and split
// once (this runs after the dependency wait, on every launch's critical
// path); WIDE: warp w splits rows g = w, w + W, ... (< 8), slot g holding
// (hi, lo) and the second-MMA register lo2.  Lane l of the warp owns the
// 4 dims 4l..4l+3 = (t, ks, half) = (l / 8, (l / 2) % 4, l % 2) of the
// fragment order described at QInt8.
template <bool WIDE>
__device__ __forceinline__ void split_q_cta(const DecodeParams& p, int r, int h, int warp,
                                            int W, int lane, QFragTable* tab) {
  const int t = lane >> 3, ks = (lane >> 1) & 3, half = lane & 1;
  constexpr int kRows = WIDE ? 8 : 4;
  for (int g = warp; g < kRows; g += W) {
    const int row = g;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (row < p.group) {
      // Rows are 4-byte aligned (the C ABI's guarantee): half2 loads.
      const __half2* q2 = reinterpret_cast<const __half2*>(
          p.q + static_cast<int64_t>(r) * p.q_stride_b +
          static_cast<int64_t>(h * p.group + row) * p.q_stride_h + 4 * lane);
      const float2 f0 = __half22float2(q2[0]);
      const float2 f1 = __half22float2(q2[1]);
      x[0] = f0.x;
      x[1] = f0.y;
      x[2] = f1.x;
      x[3] = f1.y;
    }
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sq = amax > 0.f ? amax / 127.f : 1.f;
    const float inv = 1.f / sq;
    const float inv_lo = 254.f / sq;
    const float inv_lo2 = 64516.f / sq;
    const float step_lo = sq / 254.f;
    int hv[4], lv[4], l2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int hi = clamp127(__float2int_rn(x[i] * inv));
      const float rem = fmaf(-static_cast<float>(hi), sq, x[i]);
      const int lo = clamp127(__float2int_rn(rem * inv_lo));
      const float rem2 = fmaf(-static_cast<float>(lo), step_lo, rem);
      hv[i] = hi;
      lv[i] = lo;
      l2[i] = clamp127(__float2int_rn(rem2 * inv_lo2));
    }
    const uint32_t ph = pack_s8x4(hv[0], hv[1], hv[2], hv[3]);
    const uint32_t pl = pack_s8x4(lv[0], lv[1], lv[2], lv[3]);
    const uint32_t p2 = pack_s8x4(l2[0], l2[1], l2[2], l2[3]);
    uint32_t* a = tab->a[4 * g + t] + 4 * ks + 2 * half;
    a[0] = ph;
    a[1] = pl;
    if constexpr (WIDE) {
      tab->a2[4 * g + t][2 * ks + half] = p2;
    } else {
      uint32_t* b = tab->a[4 * (g + 4) + t] + 4 * ks + 2 * half;
      b[0] = p2;
      b[1] = 0u;
    }
    if ((lane & 7) == 0) {
      tab->c[4 * g + t] = row >= p.group ? 0.f : sq * (p.sm_scale_log2 / 64516.f);
      if constexpr (!WIDE) tab->c[4 * (g + 4) + t] = 0.f;
    }
  }
  __syncthreads();
}

// This lane's query fragments from the CTA's table.
template <bool WIDE>
__device__ __forceinline__ void load_q_frag(const QFragTable* tab, int lane, QInt8<WIDE>& qi) {
  const uint4* a = reinterpret_cast<const uint4*>(tab->a[lane]);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint4 v = a[ks];
    qi.a[ks][0] = v.x;
    qi.a[ks][1] = v.y;
    qi.a[ks][2] = v.z;
    qi.a[ks][3] = v.w;
  }
  if constexpr (WIDE) {
    const uint4* a2 = reinterpret_cast<const uint4*>(tab->a2[lane]);
    const uint4 v0 = a2[0], v1 = a2[1];
    qi.a2[0][0] = v0.x;
    qi.a2[0][1] = v0.y;
    qi.a2[1][0] = v0.z;
    qi.a2[1][1] = v0.w;
    qi.a2[2][0] = v1.x;
    qi.a2[2][1] = v1.y;
    qi.a2[3][0] = v1.z;
    qi.a2[3][1] = v1.w;
  }
  qi.c = tab->c[lane];
}

__device__ __forceinline__ void mma_s8_16832(int* d, const uint32_t* a,
                                             uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// INT8 QK scores of one page for query row g: K tile at stage (16 rows of
// 128 bytes, 128B-swizzled by row) is the B operand straight from shared
// memory (n-tile 0 = tokens 0-7, n-tile 1 = tokens 8-15); the accumulator
// rows g / g+8 carry the hi / lo parts and the lo2 part comes from lane
// g+4 (GQA <= 4) or from the second mma (WIDE).  s[] = tokens 2t, 2t+1,
// 8+2t, 9+2t in log2 units (masked tokens -inf); 0 on lanes that hold no
// query row.  The int32 sums are exact; (hi*254 + lo) stays below 2^30 and
// its FP32 product with 254 rounds at 2^-24 relative.
template <bool WIDE>
__device__ __forceinline__ void qk_int8(const uint8_t* stage, const QInt8<WIDE>& qi,
                                        float sk, int valid, int g, int t,
                                        float* s) {
  const uint32_t rg = g * 128;
  const uint32_t rh = (g + 8) * 128;
  const uint32_t c0 = static_cast<uint32_t>((2 * t) ^ g) << 4;
  const uint32_t c1 = static_cast<uint32_t>((2 * t + 1) ^ g) << 4;
  const uint4 kg0 = lds128(stage, rg + c0);
  const uint4 kg1 = lds128(stage, rg + c1);
  const uint4 kh0 = lds128(stage, rh + c0);
  const uint4 kh1 = lds128(stage, rh + c1);
  int c_lo[4] = {0, 0, 0, 0}, c_hi[4] = {0, 0, 0, 0};  // n-tile 0 / 1
  mma_s8_16832(c_lo, qi.a[0], kg0.x, kg0.y);
  mma_s8_16832(c_hi, qi.a[0], kh0.x, kh0.y);
  mma_s8_16832(c_lo, qi.a[1], kg0.z, kg0.w);
  mma_s8_16832(c_hi, qi.a[1], kh0.z, kh0.w);
  mma_s8_16832(c_lo, qi.a[2], kg1.x, kg1.y);
  mma_s8_16832(c_hi, qi.a[2], kh1.x, kh1.y);
  mma_s8_16832(c_lo, qi.a[3], kg1.z, kg1.w);
  mma_s8_16832(c_hi, qi.a[3], kh1.z, kh1.w);
  int x[4];  // lo2 products of tokens 2t, 2t+1, 8+2t, 9+2t
  if constexpr (WIDE) {
    int d_lo[4] = {0, 0, 0, 0}, d_hi[4] = {0, 0, 0, 0};
    uint32_t a2[4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      a2[0] = qi.a2[ks][0];
      a2[1] = 0u;
      a2[2] = qi.a2[ks][1];
      a2[3] = 0u;
      const uint4& kg = ks < 2 ? kg0 : kg1;
      const uint4& kh = ks < 2 ? kh0 : kh1;
      mma_s8_16832(d_lo, a2, (ks & 1) ? kg.z : kg.x, (ks & 1) ? kg.w : kg.y);
      mma_s8_16832(d_hi, a2, (ks & 1) ? kh.z : kh.x, (ks & 1) ? kh.w : kh.y);
    }
    x[0] = d_lo[0];
    x[1] = d_lo[1];
    x[2] = d_hi[0];
    x[3] = d_hi[1];
  } else {
    x[0] = __shfl_down_sync(0xffffffffu, c_lo[0], 16);
    x[1] = __shfl_down_sync(0xffffffffu, c_lo[1], 16);
    x[2] = __shfl_down_sync(0xffffffffu, c_hi[0], 16);
    x[3] = __shfl_down_sync(0xffffffffu, c_hi[1], 16);
  }
  const float e = qi.c * sk;
  s[0] = fmaf(static_cast<float>(c_lo[0] * 254 + c_lo[2]), 254.f, static_cast<float>(x[0])) * e;
  s[1] = fmaf(static_cast<float>(c_lo[1] * 254 + c_lo[3]), 254.f, static_cast<float>(x[1])) * e;
  s[2] = fmaf(static_cast<float>(c_hi[0] * 254 + c_hi[2]), 254.f, static_cast<float>(x[2])) * e;
  s[3] = fmaf(static_cast<float>(c_hi[1] * 254 + c_hi[3]), 254.f, static_cast<float>(x[3])) * e;
  if (valid < kPage) {
    if (2 * t >= valid) s[0] = kNegInf;
    if (2 * t + 1 >= valid) s[1] = kNegInf;
    if (2 * t + 8 >= valid) s[2] = kNegInf;
    if (2 * t + 9 >= valid) s[3] = kNegInf;
  }
}

// Online softmax for query row g over NP pages (INT8 path).  The reference
// max m0 / sum l0 of row g live in the four lanes of groupID g.  The
// output accumulator holds rows 2t / 2t+1, whose rescale factors are
// fetched from those rows' lanes on the (rare) rescale path.
template <int NP>
__device__ __forceinline__ void softmax_rowg(WarpState& st, const float* s,
                                             const float* r, int t,
                                             uint32_t* pb0, uint32_t* pb1) {
  float lm = s[0];
#pragma unroll
  for (int i = 1; i < 4 * NP; ++i) lm = fmaxf(lm, s[i]);
  if (__any_sync(0xffffffffu, lm > st.m0 + kRescaleSlack)) {
    lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 1));
    lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 2));
    const float mn = fmaxf(st.m0, lm);
    const float a = mn == kNegInf ? 1.f : fast_exp2(st.m0 - mn);  // -inf -> 0
    st.l0 *= a;
    st.m0 = mn;
    const float a0 = __shfl_sync(0xffffffffu, a, 8 * t);
    const float a1 = __shfl_sync(0xffffffffu, a, 8 * t + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st.o[4 * i + 0] *= a0;
      st.o[4 * i + 1] *= a1;
      st.o[4 * i + 2] *= a0;
      st.o[4 * i + 3] *= a1;
    }
    st.o1[0] *= a0;
    st.o1[1] *= a1;
    st.o1[2] *= a0;
    st.o1[3] *= a1;
  }
  const float ref = st.m0 == kNegInf ? 0.f : st.m0;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const float p0 = fast_exp2(s[4 * i + 0] - ref);
    const float p1 = fast_exp2(s[4 * i + 1] - ref);
    const float p2 = fast_exp2(s[4 * i + 2] - ref);
    const float p3 = fast_exp2(s[4 * i + 3] - ref);
    st.l0 += (p0 + p1) + (p2 + p3);
    pb0[i] = pack_half2(p0 * r[i], p1 * r[i]);
    pb1[i] = pack_half2(p2 * r[i], p3 * r[i]);
  }
}

// INT8 PV of one page: V tile at stage + 2048.  ldmatrix.trans on the
// 16-bit view of the tile hands each lane the byte pairs (dims 2d, 2d+1) of
// tokens (2t, 2t+1) (and +8), so one bitwise select per register yields
// the FP16 A operand of O^T += V^T P^T for m-tile i: row g = dim 16i+2g,
// row g+8 = dim 16i+2g+1.  The PV mma runs on the biased codes z + 1152
// (exact); the bias is removed once at the end through the "ones" row
// that accumulates sum(P).  vaddr[k] = this lane's ldmatrix row offset for
// the m-tile pair {2k, 2k+1}.
__device__ __forceinline__ void pv_int8(WarpState& st, const uint8_t* stage,
                                        const uint32_t* vaddr, uint32_t pb0,
                                        uint32_t pb1, int g) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t r0, r1, r2, r3;  // (tok 0-7, m-tile 2k) (tok 8-15, 2k) (0-7, 2k+1) (8-15, 2k+1)
    ldsm_x4_trans(stage + 2048 + vaddr[k], r0, r1, r2, r3);
    uint32_t a[4];
    a[0] = biased_half2_even(r0);
    a[1] = biased_half2_odd(r0);
    a[2] = biased_half2_even(r1);
    a[3] = biased_half2_odd(r1);
    mma_16816(st.o + 4 * (2 * k), a, pb0, pb1);
    a[0] = biased_half2_even(r2);
    a[1] = biased_half2_odd(r2);
    a[2] = biased_half2_even(r3);
    a[3] = biased_half2_odd(r3);
    mma_16816(st.o + 4 * (2 * k + 1), a, pb0, pb1);
  }
  const uint32_t one = g == 0 ? 0x3c003c00u : 0u;
  const uint32_t ones[4] = {one, 0u, one, 0u};
  mma_16816(st.o1, ones, pb0, pb1);
}

// NP INT8 pages at once: the pages' QK chains, softmax work and PV chains
// are independent, which gives each warp the instruction-level parallelism
// that a single page's dependency chain lacks.
template <int NP, bool WIDE>
__device__ __forceinline__ void pages_int8(WarpState& st,
                                           const uint8_t* const* stages,
                                           const QInt8<WIDE>& qi, const float* sk,
                                           const float* r, const int* valid,
                                           int g, int t, const uint32_t* vaddr) {
  float s[4 * NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) qk_int8(stages[i], qi, sk[i], valid[i], g, t, s + 4 * i);
  uint32_t pb0[NP], pb1[NP];
  softmax_rowg<NP>(st, s, r, t, pb0, pb1);
#pragma unroll
  for (int i = 0; i < NP; ++i) pv_int8(st, stages[i], vaddr, pb0[i], pb1[i], g);
}

// INT8 pages of one warp, two at a time.  The 4-stage ring is used as two
// pair slots, each with one mbarrier that completes when both pages' K and
// V tiles have landed (one wait per pair), and one elected lane issues a
// pair's four tile copies.  When the warp's pages fit the id window (<= 64)
// the V-scale reference s_ref is the maximum over all of them, known before
// the first page, so P * s_V / s_ref never needs a mid-stream rescale and
// the ratios sit in the window; longer runs raise s_ref as they go.
__device__ __forceinline__ void issue_pair_int8(const CUtensorMap* tk, const CUtensorMap* tv,
                                                uint8_t* dst, uint64_t* bar, int n, int id0,
                                                int id1, int h) {
  const uint64_t pol = l2_evict_first_policy();
  mbar_arrive_expect_tx(bar, n * 4096);
  tma_load_3d_hint(dst, tk, 0, h, id0 * kPage, bar, pol);
  tma_load_3d_hint(dst + 2048, tv, 0, h, id0 * kPage, bar, pol);
  if (n == 2) {
    tma_load_3d_hint(dst + 4096, tk, 0, h, id1 * kPage, bar, pol);
    tma_load_3d_hint(dst + 6144, tv, 0, h, id1 * kPage, bar, pol);
  }
}

template <bool WIDE>
__device__ __forceinline__ bool run_warp_pages_int8(
    const DecodeParams& p, const CUtensorMap* tk, const CUtensorMap* tv,
    WarpState& st, uint8_t* ring, uint64_t* bars, QFragTable* qtab, QInt8<WIDE>& qi, int r,
    int h, int idx_begin, int n_pages, bool has_last, int warp, int W,
    int lane) {
  const int g = lane >> 2, t = lane & 3;
  const SegmentDesc& sd = p.seg[0];
  // A warp without pages still takes part in the CTA's query split below.
  const int n_w = n_pages > warp ? (n_pages - warp + W - 1) / W : 0;
  const int n_pairs = (n_w + 1) >> 1;

  PageWindow win;
  win.base = 0;
  win.two = n_w > 32;
  // Page ids first: they gate the prologue's tile copies.
  load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 0, lane, win.id_a, win.sk_a,
                     win.sv_a);
  win.id_b = 0;
  win.sk_b = win.sv_b = 0.f;
  if (win.two)
    load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 32, lane, win.id_b, win.sk_b,
                       win.sv_b);

  // The page ids come from the plan.  With p.int8_after_wait the pages'
  // codes and scales (written by an append that may still be running) are
  // read only after the previous kernel in the stream has completed.
  if (p.int8_after_wait) pdl_wait_primary();
  // Prologue: pairs 0 and 1 (pages 0-3).
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if (q < n_pairs) {
      const int u = 2 * q;
      const int n = u + 1 < n_w ? 2 : 1;
      const int id0 = win_id(win, u);
      const int id1 = win_id(win, n == 2 ? u + 1 : u);
      if (lane == 0) issue_pair_int8(tk, tv, ring + q * 8192, bars + q, n, id0, id1, h);
    }
  }
  // The scales travel while the first tiles are in flight.
  load_window_scales(p, sd, n_w, h, 0, lane, win.id_a, win.sk_a, win.sv_a);
  if (win.two) load_window_scales(p, sd, n_w, h, 32, lane, win.id_b, win.sk_b, win.sv_b);

  uint32_t vaddr[4];
  {
    const int j = lane >> 3, row = lane & 7;
    const int tok = 8 * (j & 1) + row;
#pragma unroll
    for (int k = 0; k < 4; ++k) vaddr[k] = tok * 128 + (((2 * k + (j >> 1)) ^ row) << 4);
  }
  pdl_wait_primary();
  split_q_cta<WIDE>(p, r, h, warp, W, lane, qtab);
  if (n_w == 0) return true;
  int last_valid = kPage;
  if (has_last) {
    const int lv = __ldg(sd.last_len + r);
    last_valid = lv < 1 ? 1 : (lv > kPage ? kPage : lv);
  }
  // The warp's last page is the request's last page when it is the item's.
  const bool last_here = has_last && warp + W * (n_w - 1) == n_pages - 1;
  load_q_frag<WIDE>(qtab, lane, qi);

  // V-scale reference and per-page ratios s_V / s_ref.
  const bool fixed_ref = n_w <= 64;
  if (fixed_ref) {
    float m = fmaxf(win.sv_a, win.sv_b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    st.sref = m;
    const float inv = m > 0.f ? 1.f / m : 1.f;
    win.sv_a = m > 0.f ? win.sv_a * inv : 1.f;
    win.sv_b = m > 0.f ? win.sv_b * inv : 1.f;
  } else {
    st.sref = win_f(win, win.sv_a, win.sv_b, 0);
  }

  bool ok = true;
  int q = 0;
  for (; q < n_pairs; ++q) {
    const int u = 2 * q;
    const bool two = u + 1 < n_w;
    const bool waited = mbar_wait_bounded(bars + (q & 1), static_cast<uint32_t>(q >> 1) & 1u);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = false;
      break;
    }
    const uint8_t* stg[2] = {ring + (q & 1) * 8192, ring + (q & 1) * 8192 + 4096};
    float sk[2], rr[2];
    int valid[2] = {kPage, kPage};
    sk[0] = win_f(win, win.sk_a, win.sk_b, u - win.base);
    sk[1] = win_f(win, win.sk_a, win.sk_b, (two ? u + 1 : u) - win.base);
    if (fixed_ref) {
      rr[0] = win_f(win, win.sv_a, win.sv_b, u - win.base);
      rr[1] = win_f(win, win.sv_a, win.sv_b, (two ? u + 1 : u) - win.base);
    } else {
      const float sv0 = win_f(win, win.sv_a, win.sv_b, u - win.base);
      const float sv1 = win_f(win, win.sv_a, win.sv_b, (two ? u + 1 : u) - win.base);
      const float svmax = fmaxf(sv0, sv1);
      if (svmax > st.sref) {
        // Keep P * (s_V / s_ref) <= P in FP16 by raising the reference.
        const float f = st.sref / svmax;
#pragma unroll
        for (int i = 0; i < 32; ++i) st.o[i] *= f;
#pragma unroll
        for (int i = 0; i < 4; ++i) st.o1[i] *= f;
        st.sref = svmax;
      }
      const float inv_ref = st.sref > 0.f ? __fdividef(1.f, st.sref) : 1.f;
      rr[0] = st.sref > 0.f ? sv0 * inv_ref : 1.f;
      rr[1] = st.sref > 0.f ? sv1 * inv_ref : 1.f;
    }
    if (last_here && q == n_pairs - 1) {
      if (two)
        valid[1] = last_valid;
      else
        valid[0] = last_valid;
    }
    if (two)
      pages_int8<2, WIDE>(st, stg, qi, sk, rr, valid, g, t, vaddr);
    else
      pages_int8<1, WIDE>(st, stg, qi, sk, rr, valid, g, t, vaddr);
    __syncwarp();
    // Refill this pair slot with pair q + 2.
    const int nq = q + 2;
    if (nq < n_pairs) {
      const int nu = 2 * nq;
      const int n = nu + 1 < n_w ? 2 : 1;
      const int id0 = win_id(win, nu);
      const int id1 = win_id(win, n == 2 ? nu + 1 : nu);
      if (lane == 0) issue_pair_int8(tk, tv, ring + (q & 1) * 8192, bars + (q & 1), n, id0, id1, h);
    }
    // Slide the id window once the consumer leaves its first half (the
    // refill above may read up to 3 pages ahead of the consumer).
    if (win.two && u + 2 - win.base >= 32) {
      win.base += 32;
      win.id_a = win.id_b;
      win.sk_a = win.sk_b;
      win.sv_a = win.sv_b;
      load_window_set<0>(p, sd, idx_begin, warp, W, n_w, h, win.base + 32, lane, win.id_b,
                         win.sk_b, win.sv_b);
    }
  }
  if (!ok) {
    record_error(p.error_flag, kDevWaitTimeout);
    // Drain copies still in flight into this warp's ring before exiting.
    const int issued_end = q + 2 < n_pairs ? q + 2 : n_pairs;
    for (int v = q; v < issued_end; ++v)
      mbar_wait_bounded(bars + (v & 1), static_cast<uint32_t>(v >> 1) & 1u);
  }
  return ok;
}

}  // namespace pg
