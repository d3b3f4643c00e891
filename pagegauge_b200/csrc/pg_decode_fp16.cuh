// FP16 pages of the split-KV decode (segment 1: the centred exact tail
// ring, or a plain FP16 cache): Q fragments, one page's QK / softmax / PV
// on FP16 tensor-core MMAs, and the per-warp TMA pipeline over the pages.
#pragma once

#include "pg_decode_core.cuh"

namespace pg {

// FP16 Q^T fragments (mma B operand) for the FP16 segment, with the same
// dimension permutation the K fragments use.
__device__ __forceinline__ void load_q_fp16(const DecodeParams& p, int r, int h,
                                            int g, int t, uint32_t* qf) {
  if (g >= p.group) {
#pragma unroll
    for (int i = 0; i < 16; ++i) qf[i] = 0u;
    return;
  }
  const uint32_t* q32 = reinterpret_cast<const uint32_t*>(
      p.q + static_cast<int64_t>(r) * p.q_stride_b +
      static_cast<int64_t>(h * p.group + g) * p.q_stride_h);
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

// One FP16 page: K dims 0-63 at st_addr, 64-127 at +2048; V likewise at
// +4096 / +6144.  Each region is 16 rows of 128 bytes, 128B-swizzled.
__device__ __forceinline__ void page_fp16(WarpState& st, const uint8_t* stage,
                                          const uint32_t* qf, float sscale,
                                          int valid, int g, int t, int group) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int R = t >> 1;
    const int cb = 4 * (t & 1);
    const uint32_t rg = R * 2048 + g * 128;
    const uint32_t rh = rg + 8 * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t c = static_cast<uint32_t>(cb + ((j + 2 * R) & 3));
      const uint32_t off = (c ^ static_cast<uint32_t>(g)) << 4;
      const uint4 kg = lds128(stage, rg + off);
      const uint4 kh = lds128(stage, rh + off);
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
  const float one_r = 1.f;
  softmax_pages<1>(st, s, &one_r, g, t, group, &pb0, &pb1);
  {
    const uint32_t ta = 2 * t, tb = 2 * t + 1;
#pragma unroll
    for (int R = 0; R < 2; ++R) {
      const uint32_t vbase = 4096 + R * 2048;
      const uint4 va = lds128(stage, vbase + ta * 128 + ((g ^ ta) << 4));
      const uint4 vb = lds128(stage, vbase + tb * 128 + ((g ^ tb) << 4));
      const uint4 vc = lds128(stage, vbase + (ta + 8) * 128 + ((g ^ ta) << 4));
      const uint4 vd = lds128(stage, vbase + (tb + 8) * 128 + ((g ^ tb) << 4));
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

// Issue the TMA copies of FP16 warp-page u into ring stage `stage` (8 KB:
// K dims 0-63 / 64-127, then V likewise).
__device__ __forceinline__ void issue_page_fp16(const CUtensorMap* tk, const CUtensorMap* tv,
                                                uint8_t* ring, uint64_t* bars, int stage, int id,
                                                int h) {
  uint8_t* dst = ring + stage * 8192;
  uint64_t* bar = bars + stage;
  const uint64_t pol = l2_evict_first_policy();
  mbar_arrive_expect_tx(bar, 8192);
  tma_load_3d_hint(dst, tk, 0, 2 * h, id * kPage, bar, pol);
  tma_load_3d_hint(dst + 2048, tk, 0, 2 * h + 1, id * kPage, bar, pol);
  tma_load_3d_hint(dst + 4096, tv, 0, 2 * h, id * kPage, bar, pol);
  tma_load_3d_hint(dst + 6144, tv, 0, 2 * h + 1, id * kPage, bar, pol);
}

// FP16 pages (the exact tail ring, or a plain FP16 cache) of one warp, one
// at a time through a 2-stage ring of 8 KB stages.
__device__ __forceinline__ bool run_warp_pages_fp16(
    const DecodeParams& p, const CUtensorMap* tk, const CUtensorMap* tv,
    WarpState& st, uint8_t* ring, uint64_t* bars, uint32_t* qf, int r,
    int h, int idx_begin, int n_pages, bool has_last, int warp, int W,
    int lane) {
  constexpr int S = kStagesI8 / 2;
  constexpr int STAGE_BYTES = 8192;
  const int g = lane >> 2, t = lane & 3;
  const SegmentDesc& sd = p.seg[1];
  const int n_w = n_pages > warp ? (n_pages - warp + W - 1) / W : 0;
  if (n_w == 0) return true;

  // Programmatic dependent launch: the FP16 exact pages may have been
  // written by the kernel just before this one (the append), so their loads
  // wait for it.
  pdl_wait_primary();

  PageWindow win;
  win.base = 0;
  win.two = n_w > 32;
  load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 0, lane, win.id_a,
                     win.sk_a, win.sv_a);
  win.id_b = 0;
  win.sk_b = win.sv_b = 0.f;
  if (win.two)
    load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 32, lane, win.id_b,
                       win.sk_b, win.sv_b);

  // Prologue: fill the ring.
  const int pro = n_w < S ? n_w : S;
  for (int u = 0; u < pro; ++u) {
    const int id = win_id(win, u);
    if (lane == 0) issue_page_fp16(tk, tv, ring, bars, u, id, h);
  }
  int last_valid = kPage;
  if (has_last) {
    const int lv = __ldg(sd.last_len + r);
    last_valid = lv < 1 ? 1 : (lv > kPage ? kPage : lv);
  }
  // Prepare Q while the first tiles are in flight.
  load_q_fp16(p, r, h, g, t, qf);
  bool ok = true;
  int u = 0;
  while (u < n_w) {
    const bool waited = mbar_wait_bounded(bars + (u % S), static_cast<uint32_t>(u / S) & 1u);
    if (!__all_sync(0xffffffffu, waited)) {
      ok = false;
      break;
    }
    const int valid = (has_last && warp + W * u == n_pages - 1) ? last_valid : kPage;
    page_fp16(st, ring + (u % S) * STAGE_BYTES, qf, p.sm_scale_log2, valid, g, t, p.group);
    __syncwarp();
    const int nu = u + S;
    if (nu < n_w) {
      const int id = win_id(win, nu);
      if (lane == 0) issue_page_fp16(tk, tv, ring, bars, u % S, id, h);
    }
    u += 1;
    // Slide the id window once the consumer leaves its first half.
    if (win.two && u - win.base >= 32) {
      win.base += 32;
      win.id_a = win.id_b;
      load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, win.base + 32,
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

}  // namespace pg
