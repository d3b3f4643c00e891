// Split-KV paged GQA decode attention over PageGauge caches (sm_100a).
//
// One CTA processes one work item: (request, KV head, segment, contiguous
// run of that request's logical pages).  Segment 0 holds completed pages as
// signed INT8 codes with one FP16 scale per (page, KV head); segment 1 holds
// centred FP16 pages (the exact tail ring, or a plain FP16 cache).
//
// Inside a CTA every warp owns an independent TMA pipeline: it takes every
// W-th page of the item, stages the page's K and V tiles (16 tokens x 128
// dims of one KV head) into a private shared-memory ring with a 3-D tiled
// bulk-tensor copy (128-byte swizzle), and computes
//   S^T = K_tile (16 tok x 128) . Q^T (128 x 8 q-rows)   (8 mma.sync)
//   O^T += V_tile^T (128 x 16 tok) . P^T (16 tok x 8)     (8 mma.sync)
// with the GQA group (<= 8 query heads sharing the KV head) in the N=8
// columns.  INT8 codes become FP16 in registers with an exact
// byte-permute + one f16x2 subtraction; the page K scale is applied to the
// fp32 scores after the MMA and the page V scale to the probabilities
// before the PV MMA, the factorisation PageGauge uses (c_K cancels in the
// softmax, c_V is restored once after normalisation).
//
// Online softmax is in base 2 (scores scaled by sm_scale*log2(e)); the log-
// sum-exp written for a partial state is base 2 as well.
#pragma once

#include "pg_common.cuh"

namespace pg {

// 16-byte work item (host builds the list in plan()).
struct DecodeItem {
  int32_t request;
  int32_t head_seg;   // kv head in the low 16 bits, segment in the high 16
  int32_t idx_begin;  // absolute offset of the item's first page id
  int32_t count;      // pages in the item; bit 31 set: contains the
                      // request's last page (masked by last_page_len)
};

struct SegmentDesc {
  const int32_t* indices;   // physical page ids
  const int32_t* last_len;  // [B] tokens in each request's last page
  const __half* k_scale;    // [pages, Hkv] (INT8 segment only)
  const __half* v_scale;
  int32_t num_pages;        // pages allocated in the cache tensor
};

struct DecodeParams {
  const __half* q;
  int64_t q_stride_b, q_stride_h;
  SegmentDesc seg[2];
  const DecodeItem* items;
  int32_t num_items;
  int32_t hkv;
  int32_t group;
  float sm_scale_log2;
  // Partial epilogue: normalised partial output and base-2 lse per item.
  float* part_o;    // [num_items, group, 128]
  float* part_lse;  // [num_items, group]
  // Final epilogue (exactly one item per (request, kv head)).
  int32_t final_mode;
  __half* out;
  int64_t out_stride_b, out_stride_h;
  float* lse_out;  // [B, Hq] or null
  const __half* extra_o;  // optional state merged in (may alias out)
  int64_t extra_stride_b, extra_stride_h;
  const float* extra_lse;  // [B, Hq] (may alias lse_out)
  const __half* value_center;  // [B, Hkv, 128] or null
  int64_t vc_stride_b;         // 0 broadcasts one [Hkv,128] centre
  // items == null: implicit list, CTA b = (request b / Hkv, head b % Hkv)
  // over `implicit_pages` FP16 pages starting at request * implicit_pages.
  int32_t implicit_pages;
  int* error_flag;
};

constexpr int kStagesI8 = 4;              // INT8 stages per warp
constexpr int kRingBytes = kStagesI8 * 4096;
constexpr int kMaxWarps = 8;

__host__ __device__ constexpr int decode_smem_bytes(int warps) {
  return warps * kRingBytes + warps * kStagesI8 * 8 + 1024;
}

// Output dimension held by accumulator row (m-tile i, row g / g+8).
template <int SEG>
__device__ __forceinline__ int out_dim(int i, int g, int odd) {
  if (SEG == 0) return 16 * g + 2 * i + odd;
  return 64 * (i >> 2) + 8 * g + 2 * (i & 3) + odd;
}

struct WarpState {
  float m0, m1, l0, l1;
  float o[32];
  float sref;
};

// Page-id / scale window: lane L of set A holds warp-page base+L, set B
// holds base+32+L.  Shuffles fetch the value of any page in [base, base+64).
struct PageWindow {
  int base;
  int id_a, id_b;
  float sk_a, sk_b, sv_a, sv_b;
};

template <int SEG>
__device__ __forceinline__ void load_window_set(const DecodeParams& p,
                                                const SegmentDesc& sd,
                                                int idx_begin, int warp, int W,
                                                int n_w, int h, int first,
                                                int lane, int& id, float& sk,
                                                float& sv) {
  const int u = first + lane;
  id = 0;
  sk = 0.f;
  sv = 0.f;
  if (u < n_w) {
    id = __ldg(sd.indices + idx_begin + warp + W * u);
    if (id < 0 || id >= sd.num_pages) {
      record_error(p.error_flag, kDevBadPageId);
      id = 0;
    }
    if (SEG == 0) {
      sk = __half2float(sd.k_scale[static_cast<int64_t>(id) * p.hkv + h]);
      sv = __half2float(sd.v_scale[static_cast<int64_t>(id) * p.hkv + h]);
    }
  }
}

__device__ __forceinline__ int win_id(const PageWindow& w, int u) {
  const int k = u - w.base;
  const int a = __shfl_sync(0xffffffffu, w.id_a, k & 31);
  const int b = __shfl_sync(0xffffffffu, w.id_b, k & 31);
  return k < 32 ? a : b;
}
__device__ __forceinline__ float win_f(float fa, float fb, int k) {
  const float a = __shfl_sync(0xffffffffu, fa, k & 31);
  const float b = __shfl_sync(0xffffffffu, fb, k & 31);
  return k < 32 ? a : b;
}

// Q^T fragments (mma B operand) with the same dimension permutation the K
// fragments use, so the contraction over head_dim is unchanged.
template <int SEG>
__device__ __forceinline__ void load_q_frag(const DecodeParams& p, int r,
                                            int h, int g, int t,
                                            uint32_t* qf) {
  if (g >= p.group) {
#pragma unroll
    for (int i = 0; i < 16; ++i) qf[i] = 0u;
    return;
  }
  const __half* qrow =
      p.q + static_cast<int64_t>(r) * p.q_stride_b +
      static_cast<int64_t>(h * p.group + g) * p.q_stride_h;
  const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qrow);
  if (SEG == 0) {
    // thread t covers dims [32t, 32t+32); k-step ks uses dims 32t+4ks..+3
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qf[2 * ks] = __ldg(q32 + (32 * t + 4 * ks) / 2);
      qf[2 * ks + 1] = __ldg(q32 + (32 * t + 4 * ks + 2) / 2);
    }
  } else {
    const int R = t >> 1;
    const int cb = 4 * (t & 1);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int j = ks >> 1, e = ks & 1;
      const int c = cb + ((j + 2 * R) & 3);
      const int d = 64 * R + 8 * c + 4 * e;
      qf[2 * ks] = __ldg(q32 + d / 2);
      qf[2 * ks + 1] = __ldg(q32 + (d + 2) / 2);
    }
  }
}

// Online-softmax update for one 16-token page given raw fp32 scores.
// Returns the packed P^T fragments (pb0, pb1) for the PV mma.
__device__ __forceinline__ void softmax_page(WarpState& st, float* s, float r,
                                             int g, int t, int group,
                                             uint32_t& pb0, uint32_t& pb1) {
  float mx0 = warp_max_xor_g(fmaxf(s[0], s[2]));
  float mx1 = warp_max_xor_g(fmaxf(s[1], s[3]));
  const float mn0 = fmaxf(st.m0, mx0);
  const float mn1 = fmaxf(st.m1, mx1);
  const float ref0 = mn0 == kNegInf ? 0.f : mn0;
  const float ref1 = mn1 == kNegInf ? 0.f : mn1;
  const float a0 = fast_exp2(st.m0 - ref0);
  const float a1 = fast_exp2(st.m1 - ref1);
  const float p0 = fast_exp2(s[0] - ref0);
  const float p1 = fast_exp2(s[1] - ref1);
  const float p2 = fast_exp2(s[2] - ref0);
  const float p3 = fast_exp2(s[3] - ref1);
  st.l0 = st.l0 * a0 + (p0 + p2);
  st.l1 = st.l1 * a1 + (p1 + p3);
  st.m0 = mn0;
  st.m1 = mn1;
  // Rescale the running output only when some row's maximum moved.
  if (__any_sync(0xffffffffu, (a0 != 1.f) || (a1 != 1.f))) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st.o[4 * i + 0] *= a0;
      st.o[4 * i + 1] *= a1;
      st.o[4 * i + 2] *= a0;
      st.o[4 * i + 3] *= a1;
    }
  }
  const uint32_t h01 = pack_half2(p0 * r, p1 * r);
  const uint32_t h23 = pack_half2(p2 * r, p3 * r);
  const int src0 = 8 * t + (g >> 1);
  const int src1 = src0 + 4;
  const uint32_t x01 = __shfl_sync(0xffffffffu, h01, src0);
  const uint32_t y01 = __shfl_sync(0xffffffffu, h01, src1);
  const uint32_t x23 = __shfl_sync(0xffffffffu, h23, src0);
  const uint32_t y23 = __shfl_sync(0xffffffffu, h23, src1);
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
  pb0 = prmt(x01, y01, sel);
  pb1 = prmt(x23, y23, sel);
  if (g >= group) {
    pb0 = 0u;
    pb1 = 0u;
  }
}

// One INT8 page: K tile at st_addr, V tile at st_addr + 2048 (both 16 rows
// of 128 bytes, 128B-swizzled by row).
__device__ __forceinline__ void page_int8(WarpState& st, uint32_t st_addr,
                                          const uint32_t* qf, float kscale,
                                          float r, int valid, int g, int t,
                                          int group) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint32_t rg = st_addr + g * 128;
    const uint32_t rh = st_addr + (g + 8) * 128;
    const uint32_t c0 = static_cast<uint32_t>((2 * t) ^ g) << 4;
    const uint32_t c1 = static_cast<uint32_t>((2 * t + 1) ^ g) << 4;
    const uint4 kg0 = lds128(rg + c0);
    const uint4 kg1 = lds128(rg + c1);
    const uint4 kh0 = lds128(rh + c0);
    const uint4 kh1 = lds128(rh + c1);
    const uint32_t wg[8] = {kg0.x, kg0.y, kg0.z, kg0.w,
                            kg1.x, kg1.y, kg1.z, kg1.w};
    const uint32_t wh[8] = {kh0.x, kh0.y, kh0.z, kh0.w,
                            kh1.x, kh1.y, kh1.z, kh1.w};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t xg = wg[ks] ^ 0x80808080u;
      const uint32_t xh = wh[ks] ^ 0x80808080u;
      uint32_t a[4];
      a[0] = hsub2_u32(prmt(xg, kMagic, 0x4140u), kBias2);
      a[1] = hsub2_u32(prmt(xh, kMagic, 0x4140u), kBias2);
      a[2] = hsub2_u32(prmt(xg, kMagic, 0x4342u), kBias2);
      a[3] = hsub2_u32(prmt(xh, kMagic, 0x4342u), kBias2);
      mma_16816(s, a, qf[2 * ks], qf[2 * ks + 1]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] *= kscale;
  if (valid < kPage) {
    if (g >= valid) s[0] = s[1] = kNegInf;
    if (g + 8 >= valid) s[2] = s[3] = kNegInf;
  }
  uint32_t pb0, pb1;
  softmax_page(st, s, r, g, t, group, pb0, pb1);
  {
    const uint32_t vbase = st_addr + 2048;
    const uint32_t ta = 2 * t, tb = 2 * t + 1;
    const uint4 va = lds128(vbase + ta * 128 + ((g ^ ta) << 4));
    const uint4 vb = lds128(vbase + tb * 128 + ((g ^ tb) << 4));
    const uint4 vc = lds128(vbase + (ta + 8) * 128 + ((g ^ ta) << 4));
    const uint4 vd = lds128(vbase + (tb + 8) * 128 + ((g ^ tb) << 4));
    const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
    const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
    const uint32_t wc[4] = {vc.x, vc.y, vc.z, vc.w};
    const uint32_t wd[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t x = wa[k] ^ 0x80808080u, y = wb[k] ^ 0x80808080u;
      const uint32_t z = wc[k] ^ 0x80808080u, w = wd[k] ^ 0x80808080u;
      const uint32_t lo_ab = prmt(x, y, 0x5140u), hi_ab = prmt(x, y, 0x7362u);
      const uint32_t lo_cd = prmt(z, w, 0x5140u), hi_cd = prmt(z, w, 0x7362u);
      uint32_t a[4];
      a[0] = hsub2_u32(prmt(lo_ab, kMagic, 0x4140u), kBias2);
      a[1] = hsub2_u32(prmt(lo_ab, kMagic, 0x4342u), kBias2);
      a[2] = hsub2_u32(prmt(lo_cd, kMagic, 0x4140u), kBias2);
      a[3] = hsub2_u32(prmt(lo_cd, kMagic, 0x4342u), kBias2);
      mma_16816(st.o + 4 * (2 * k), a, pb0, pb1);
      a[0] = hsub2_u32(prmt(hi_ab, kMagic, 0x4140u), kBias2);
      a[1] = hsub2_u32(prmt(hi_ab, kMagic, 0x4342u), kBias2);
      a[2] = hsub2_u32(prmt(hi_cd, kMagic, 0x4140u), kBias2);
      a[3] = hsub2_u32(prmt(hi_cd, kMagic, 0x4342u), kBias2);
      mma_16816(st.o + 4 * (2 * k + 1), a, pb0, pb1);
    }
  }
}

// One FP16 page: K dims 0-63 at st_addr, 64-127 at +2048; V likewise at
// +4096 / +6144.  Each region is 16 rows of 128 bytes, 128B-swizzled.
__device__ __forceinline__ void page_fp16(WarpState& st, uint32_t st_addr,
                                          const uint32_t* qf, float sscale,
                                          int valid, int g, int t, int group) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int R = t >> 1;
    const int cb = 4 * (t & 1);
    const uint32_t rg = st_addr + R * 2048 + g * 128;
    const uint32_t rh = rg + 8 * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t c = static_cast<uint32_t>(cb + ((j + 2 * R) & 3));
      const uint32_t off = (c ^ static_cast<uint32_t>(g)) << 4;
      const uint4 kg = lds128(rg + off);
      const uint4 kh = lds128(rh + off);
      uint32_t a[4];
      a[0] = kg.x;
      a[1] = kh.x;
      a[2] = kg.y;
      a[3] = kh.y;
      mma_16816(s, a, qf[4 * j], qf[4 * j + 1]);
      a[0] = kg.z;
      a[1] = kh.z;
      a[2] = kg.w;
      a[3] = kh.w;
      mma_16816(s, a, qf[4 * j + 2], qf[4 * j + 3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] *= sscale;
  if (valid < kPage) {
    if (g >= valid) s[0] = s[1] = kNegInf;
    if (g + 8 >= valid) s[2] = s[3] = kNegInf;
  }
  uint32_t pb0, pb1;
  softmax_page(st, s, 1.f, g, t, group, pb0, pb1);
  {
    const uint32_t ta = 2 * t, tb = 2 * t + 1;
#pragma unroll
    for (int R = 0; R < 2; ++R) {
      const uint32_t vbase = st_addr + 4096 + R * 2048;
      const uint4 va = lds128(vbase + ta * 128 + ((g ^ ta) << 4));
      const uint4 vb = lds128(vbase + tb * 128 + ((g ^ tb) << 4));
      const uint4 vc = lds128(vbase + (ta + 8) * 128 + ((g ^ ta) << 4));
      const uint4 vd = lds128(vbase + (tb + 8) * 128 + ((g ^ tb) << 4));
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
      const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
      const uint32_t wc[4] = {vc.x, vc.y, vc.z, vc.w};
      const uint32_t wd[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t a[4];
        a[0] = prmt(wa[k], wb[k], 0x5410u);
        a[1] = prmt(wa[k], wb[k], 0x7632u);
        a[2] = prmt(wc[k], wd[k], 0x5410u);
        a[3] = prmt(wc[k], wd[k], 0x7632u);
        mma_16816(st.o + 4 * (4 * R + k), a, pb0, pb1);
      }
    }
  }
}

// Issue the TMA copies of warp-page u into ring stage `stage`.
template <int SEG>
__device__ __forceinline__ void issue_page(const CUtensorMap* tk,
                                           const CUtensorMap* tv,
                                           uint8_t* ring, uint64_t* bars,
                                           int stage, int id, int h) {
  if (SEG == 0) {
    uint8_t* dst = ring + stage * 4096;
    uint64_t* bar = bars + stage;
    mbar_arrive_expect_tx(bar, 4096);
    tma_load_3d(dst, tk, 0, h, id * kPage, bar);
    tma_load_3d(dst + 2048, tv, 0, h, id * kPage, bar);
  } else {
    uint8_t* dst = ring + stage * 8192;
    uint64_t* bar = bars + stage;
    mbar_arrive_expect_tx(bar, 8192);
    tma_load_3d(dst, tk, 0, 2 * h, id * kPage, bar);
    tma_load_3d(dst + 2048, tk, 0, 2 * h + 1, id * kPage, bar);
    tma_load_3d(dst + 4096, tv, 0, 2 * h, id * kPage, bar);
    tma_load_3d(dst + 6144, tv, 0, 2 * h + 1, id * kPage, bar);
  }
}

template <int SEG>
__device__ __forceinline__ bool run_warp_pages(
    const DecodeParams& p, const CUtensorMap* tk, const CUtensorMap* tv,
    WarpState& st, uint8_t* ring, uint64_t* bars, const uint32_t* qf, int r,
    int h, int idx_begin, int n_pages, bool has_last, int warp, int W,
    int lane) {
  constexpr int S = SEG == 0 ? kStagesI8 : kStagesI8 / 2;
  constexpr int STAGE_BYTES = SEG == 0 ? 4096 : 8192;
  const int g = lane >> 2, t = lane & 3;
  const SegmentDesc& sd = p.seg[SEG];
  const int n_w = n_pages > warp ? (n_pages - warp + W - 1) / W : 0;
  if (n_w == 0) return true;

  int last_valid = kPage;
  if (has_last) {
    const int lv = __ldg(sd.last_len + r);
    last_valid = lv < 1 ? 1 : (lv > kPage ? kPage : lv);
  }

  PageWindow win;
  win.base = 0;
  load_window_set<SEG>(p, sd, idx_begin, warp, W, n_w, h, 0, lane, win.id_a,
                       win.sk_a, win.sv_a);
  load_window_set<SEG>(p, sd, idx_begin, warp, W, n_w, h, 32, lane, win.id_b,
                       win.sk_b, win.sv_b);

  // Prologue: fill the ring.
  const int pro = n_w < S ? n_w : S;
  for (int u = 0; u < pro; ++u) {
    const int id = win_id(win, u);
    if (lane == 0) issue_page<SEG>(tk, tv, ring, bars, u, id, h);
  }

  if (SEG == 0) st.sref = win_f(win.sv_a, win.sv_b, 0);
  bool ok = true;
  int u = 0;
  for (; u < n_w; ++u) {
    const int stage = u % S;
    const uint32_t parity = static_cast<uint32_t>(u / S) & 1u;
    const bool waited = mbar_wait_bounded(bars + stage, parity);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = false;
      break;
    }
    const int k = u - win.base;
    const int local = warp + W * u;
    const int valid = (has_last && local == n_pages - 1) ? last_valid : kPage;
    const uint32_t st_addr = smem_addr(ring + stage * STAGE_BYTES);
    if (SEG == 0) {
      const float sk = win_f(win.sk_a, win.sk_b, k);
      const float sv = win_f(win.sv_a, win.sv_b, k);
      if (sv > st.sref) {
        // Keep P * (s_V / s_ref) <= 1 in FP16 by raising the reference.
        const float f = st.sref / sv;
#pragma unroll
        for (int i = 0; i < 32; ++i) st.o[i] *= f;
        st.sref = sv;
      }
      const float rr = st.sref > 0.f ? sv / st.sref : 1.f;
      page_int8(st, st_addr, qf, sk * p.sm_scale_log2, rr, valid, g, t,
                p.group);
    } else {
      page_fp16(st, st_addr, qf, p.sm_scale_log2, valid, g, t, p.group);
    }
    __syncwarp();
    const int nu = u + S;
    if (nu < n_w) {
      const int id = win_id(win, nu);
      if (lane == 0) issue_page<SEG>(tk, tv, ring, bars, stage, id, h);
    }
    // Slide the id window once the consumer leaves its first half.
    if (u + 1 - win.base == 32) {
      win.base += 32;
      win.id_a = win.id_b;
      win.sk_a = win.sk_b;
      win.sv_a = win.sv_b;
      load_window_set<SEG>(p, sd, idx_begin, warp, W, n_w, h, win.base + 32,
                           lane, win.id_b, win.sk_b, win.sv_b);
    }
  }
  if (!ok) {
    record_error(p.error_flag, kDevWaitTimeout);
    // Drain copies still in flight into this warp's ring before exiting.
    const int issued_end = (u + S < n_w) ? u + S : n_w;
    for (int v = u; v < issued_end; ++v) {
      mbar_wait_bounded(bars + (v % S), static_cast<uint32_t>(v / S) & 1u);
    }
  }
  return ok;
}

__global__ void __launch_bounds__(kMaxWarps * 32)
    pg_decode_split_kernel(const __grid_constant__ CUtensorMap tm_k8,
                           const __grid_constant__ CUtensorMap tm_v8,
                           const __grid_constant__ CUtensorMap tm_k16,
                           const __grid_constant__ CUtensorMap tm_v16,
                           const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + W * kRingBytes);
  uint64_t* bars = bars_all + warp * kStagesI8;
  uint8_t* ring = smem + warp * kRingBytes;

  DecodeItem item;
  if (p.items != nullptr) {
    item = p.items[blockIdx.x];
  } else {
    item.request = static_cast<int>(blockIdx.x) / p.hkv;
    item.head_seg = (static_cast<int>(blockIdx.x) % p.hkv) | (1 << 16);
    item.idx_begin = item.request * p.implicit_pages;
    item.count = p.implicit_pages | static_cast<int32_t>(0x80000000u);
  }
  const int r = item.request;
  const int h = item.head_seg & 0xffff;
  const int seg = item.head_seg >> 16;
  const int n_pages = item.count & 0x7fffffff;
  const bool has_last = item.count < 0;

  if (lane == 0) {
    for (int s = 0; s < kStagesI8; ++s) mbar_init(bars + s, 1);
    fence_barrier_init();
    if (warp == 0) {
      prefetch_tensormap(seg == 0 ? &tm_k8 : &tm_k16);
      prefetch_tensormap(seg == 0 ? &tm_v8 : &tm_v16);
    }
  }
  __syncwarp();

  WarpState st;
  st.m0 = st.m1 = kNegInf;
  st.l0 = st.l1 = 0.f;
  st.sref = 1.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) st.o[i] = 0.f;

  uint32_t qf[16];
  bool ok;
  if (seg == 0) {
    load_q_frag<0>(p, r, h, g, t, qf);
    ok = run_warp_pages<0>(p, &tm_k8, &tm_v8, st, ring, bars, qf, r, h,
                           item.idx_begin, n_pages, has_last, warp, W, lane);
  } else {
    load_q_frag<1>(p, r, h, g, t, qf);
    ok = run_warp_pages<1>(p, &tm_k16, &tm_v16, st, ring, bars, qf, r, h,
                           item.idx_begin, n_pages, has_last, warp, W, lane);
  }
  // Let a dependent (merge) grid start launching while we finish.
  pdl_launch_dependents();

  // Per-warp totals: reduce l across the 8 token lanes.
  st.l0 = warp_sum_xor_g(st.l0);
  st.l1 = warp_sum_xor_g(st.l1);
  const float oscale = seg == 0 ? st.sref : 1.f;

  __syncthreads();  // every warp has drained its ring
  const int group = p.group;
  float* cm = reinterpret_cast<float*>(smem);          // [W][8]
  float* cl = cm + kMaxWarps * 8;                      // [W][8]
  float* co = cl + kMaxWarps * 8;                      // [W][8][128]
  const int q0 = 2 * t, q1 = 2 * t + 1;
  if (g == 0) {
    cm[warp * 8 + q0] = ok ? st.m0 : kNegInf;
    cm[warp * 8 + q1] = ok ? st.m1 : kNegInf;
    cl[warp * 8 + q0] = ok ? st.l0 : 0.f;
    cl[warp * 8 + q1] = ok ? st.l1 : 0.f;
  }
  if (q0 < group) {
    float* c0 = co + (warp * 8 + q0) * kHeadDim;
    float* c1 = co + (warp * 8 + q1) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int d0, d1;
      if (seg == 0) {
        d0 = out_dim<0>(i, g, 0);
        d1 = out_dim<0>(i, g, 1);
      } else {
        d0 = out_dim<1>(i, g, 0);
        d1 = out_dim<1>(i, g, 1);
      }
      c0[d0] = st.o[4 * i + 0] * oscale;
      c0[d1] = st.o[4 * i + 2] * oscale;
      if (q1 < group) {
        c1[d0] = st.o[4 * i + 1] * oscale;
        c1[d1] = st.o[4 * i + 3] * oscale;
      }
    }
  }
  __syncthreads();

  // The extra state may alias the outputs (in-place merge): read its lse
  // for every row before any thread writes lse_out.
  float* xls = co + W * 8 * kHeadDim;  // [8], inside this CTA's rings
  if (p.final_mode && p.extra_o != nullptr && threadIdx.x < group)
    xls[threadIdx.x] = p.extra_lse[static_cast<int64_t>(r) * (p.hkv * group) + h * group + threadIdx.x];
  __syncthreads();
  const int total = group * kHeadDim;
  for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
    const int q = idx >> 7, d = idx & 127;
    float M = kNegInf;
    for (int w = 0; w < W; ++w) M = fmaxf(M, cm[w * 8 + q]);
    float L = 0.f, O = 0.f;
    if (M != kNegInf) {
      for (int w = 0; w < W; ++w) {
        const float mw = cm[w * 8 + q];
        if (mw == kNegInf) continue;
        const float e = fast_exp2(mw - M);
        L += cl[w * 8 + q] * e;
        O += co[(w * 8 + q) * kHeadDim + d] * e;
      }
    }
    const float on = L > 0.f ? O / L : 0.f;
    const float lse = L > 0.f ? M + fast_log2(L) : kNegInf;
    if (!p.final_mode) {
      const int64_t base = static_cast<int64_t>(blockIdx.x) * group + q;
      p.part_o[base * kHeadDim + d] = on;
      if (d == 0) p.part_lse[base] = lse;
    } else {
      const int qh = h * group + q;
      float v = on, lv = lse;
      if (p.extra_o != nullptr) {
        const float xl = xls[q];
        const float xo = __half2float(
            p.extra_o[static_cast<int64_t>(r) * p.extra_stride_b +
                      static_cast<int64_t>(qh) * p.extra_stride_h + d]);
        const float mm = fmaxf(xl, lv);
        if (mm == kNegInf) {
          v = 0.f;
          lv = kNegInf;
        } else {
          const float wx = fast_exp2(xl - mm), wy = fast_exp2(lv - mm);
          const float den = wx + wy;
          v = (wx * xo + wy * v) / den;
          lv = mm + fast_log2(den);
        }
      }
      if (p.value_center != nullptr) {
        v += __half2float(p.value_center[static_cast<int64_t>(r) * p.vc_stride_b +
                                         h * kHeadDim + d]);
      }
      // All threads read the extra state before any thread writes: the
      // output may alias it, and (q, d) is owned by exactly this thread.
      p.out[static_cast<int64_t>(r) * p.out_stride_b +
            static_cast<int64_t>(qh) * p.out_stride_h + d] = __float2half_rn(v);
      if (d == 0 && p.lse_out != nullptr)
        p.lse_out[static_cast<int64_t>(r) * (p.hkv * group) + qh] = lv;
    }
  }
}

// --------------------------------------------------------------- merging
struct MergeParams {
  const float* part_o;
  const float* part_lse;
  const int32_t* item_off;  // [B*Hkv + 1] partial ranges per (request, head)
  int32_t batch, hkv, group;
  __half* out;
  int64_t out_stride_b, out_stride_h;
  float* lse_out;
  const __half* extra_o;
  int64_t extra_stride_b, extra_stride_h;
  const float* extra_lse;
  const __half* value_center;
  int64_t vc_stride_b;
};

// One CTA of 128 threads per (request, query head).  Warp w folds the
// partials w, w+4, ... with float4 lanes (4 dims per lane, independent
// loads in flight), then the four warp states are combined in shared
// memory and thread d writes output dim d.
__global__ void __launch_bounds__(128)
    pg_merge_partials_kernel(const __grid_constant__ MergeParams p) {
  __shared__ float s_m[4], s_den[4];
  __shared__ float4 s_acc[4][32];
  pdl_wait_primary();
  const int hq = p.hkv * p.group;
  const int r = blockIdx.x / hq;
  const int qh = blockIdx.x % hq;
  const int h = qh / p.group, q = qh % p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int begin = p.item_off[r * p.hkv + h];
  const int end = p.item_off[r * p.hkv + h + 1];
  float m = kNegInf, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto push = [&](float lse, float4 v) {
    if (lse == kNegInf) return;
    if (lse > m) {
      const float sc = fast_exp2(m - lse);  // m = -inf -> 0
      acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
      den *= sc;
      m = lse;
    }
    const float w = fast_exp2(lse - m);
    acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
    den += w;
  };
  constexpr int U = 4;
  for (int i0 = begin + warp; i0 < end; i0 += 4 * U) {
    float l[U];
    float4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int i = i0 + 4 * k;
      l[k] = kNegInf;
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < end) {
        const int64_t b = static_cast<int64_t>(i) * p.group + q;
        l[k] = p.part_lse[b];
        v[k] = reinterpret_cast<const float4*>(p.part_o + b * kHeadDim)[lane];
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) push(l[k], v[k]);
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_den[warp] = den;
  }
  s_acc[warp][lane] = acc;
  __syncthreads();
  const int d = threadIdx.x;
  float M = kNegInf;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w]);
  float D = 0.f, A = 0.f;
  if (M != kNegInf) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (s_m[w] == kNegInf) continue;
      const float e = fast_exp2(s_m[w] - M);
      D += s_den[w] * e;
      A += reinterpret_cast<const float*>(&s_acc[w][d >> 2])[d & 3] * e;
    }
  }
  float lse = D > 0.f ? M + fast_log2(D) : kNegInf;
  float v = D > 0.f ? A / D : 0.f;
  if (p.extra_o != nullptr) {
    const float xl = p.extra_lse[static_cast<int64_t>(r) * hq + qh];
    const float xo = __half2float(p.extra_o[static_cast<int64_t>(r) * p.extra_stride_b +
                                            static_cast<int64_t>(qh) * p.extra_stride_h + d]);
    const float mm = fmaxf(xl, lse);
    if (mm == kNegInf) {
      v = 0.f;
    } else {
      const float wx = fast_exp2(xl - mm), wy = fast_exp2(lse - mm);
      v = (wx * xo + wy * v) / (wx + wy);
      lse = mm + fast_log2(wx + wy);
    }
  }
  if (p.value_center != nullptr)
    v += __half2float(p.value_center[static_cast<int64_t>(r) * p.vc_stride_b + h * kHeadDim + d]);
  __syncthreads();  // out / lse_out may alias extra_o / extra_lse
  p.out[static_cast<int64_t>(r) * p.out_stride_b + static_cast<int64_t>(qh) * p.out_stride_h + d] =
      __float2half_rn(v);
  if (d == 0 && p.lse_out != nullptr) p.lse_out[static_cast<int64_t>(r) * hq + qh] = lse;
}

// merge_state_in_place: (v_a, s_a) <- merge((v_a, s_a), (v_b, s_b)).
__global__ void pg_merge_state_kernel(__half* va, float* sa, const __half* vb,
                                      const float* sb, int64_t rows,
                                      int64_t va_row_stride,
                                      int64_t vb_row_stride) {
  const int64_t row = blockIdx.x;
  const int d = threadIdx.x;
  const float la = sa[row], lb = sb[row];
  const float m = fmaxf(la, lb);
  float v, l;
  const float xa = __half2float(va[row * va_row_stride + d]);
  const float xb = __half2float(vb[row * vb_row_stride + d]);
  if (m == kNegInf) {
    v = 0.f;
    l = kNegInf;
  } else {
    const float wa = fast_exp2(la - m), wb = fast_exp2(lb - m);
    v = (wa * xa + wb * xb) / (wa + wb);
    l = m + fast_log2(wa + wb);
  }
  __syncthreads();
  va[row * va_row_stride + d] = __float2half_rn(v);
  if (d == 0) sa[row] = l;
}

}  // namespace pg
