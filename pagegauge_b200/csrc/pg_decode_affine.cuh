// affine_group16 pages of the split-KV decode (segment 0 with a per
// (page, KV head, 16-dim group) scale and bias).
#pragma once

#include "pg_decode_core.cuh"

namespace pg {

// ------------------------------------------------------- affine_group16
// The reference's alternative representation "affine_group16"
// (scripts/benchmark_flashinfer_page_affine_int8.py:234-253; its FA2
// variant :33-73 and the affine branch of compute_qk in the INT8 patch):
// per (page, KV head, 16-dim group g) an FP16 scale s_g and bias b_g with
// x ~ z * s_g + b_g, z the signed code; no centres.  As that variant does,
// K and V are rebuilt in FP16 in registers (code -> half exactly, then one
// f16x2 FMA with the group's scale and bias, a single rounding) and fed to
// FP16 MMAs with FP32 accumulation:
//   S^T = K (16 tok x 128) . Q^T   K as the A operand (ldmatrix), group c =
//                                   k-step c
//   O^T += V^T . P^T               V^T as the A operand (ldmatrix.trans),
//                                   group i = m-tile i
// The K A-fragments take dims (4t, 4t+2) for k (2t, 2t+1) and (4t+1, 4t+3)
// for k (2t+8, 2t+9) of each 16-dim chunk (the byte order one 32-bit word
// of a row holds); Q uses the same order.

// Q^T fragments (mma B operand) for the affine QK: qa[2c] = (q[16c+4t],
// q[16c+4t+2]), qa[2c+1] = (q[16c+4t+1], q[16c+4t+3]) of query row g.
__device__ __forceinline__ void load_q_affine(const DecodeParams& p, int r, int h, int g,
                                              int t, uint32_t* qa) {
  if (g >= p.group) {
#pragma unroll
    for (int i = 0; i < 16; ++i) qa[i] = 0u;
    return;
  }
  const uint32_t* q32 = reinterpret_cast<const uint32_t*>(
      p.q + static_cast<int64_t>(r) * p.q_stride_b +
      static_cast<int64_t>(h * p.group + g) * p.q_stride_h);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t w0 = __ldg(q32 + 8 * c + 2 * t);      // dims 16c+4t, +1
    const uint32_t w1 = __ldg(q32 + 8 * c + 2 * t + 1);  // dims 16c+4t+2, +3
    qa[2 * c] = prmt(w0, w1, 0x5410u);
    qa[2 * c + 1] = prmt(w0, w1, 0x7632u);
  }
}

// Half c of an 8-half metadata row, broadcast to both lanes of a half2.
__device__ __forceinline__ uint32_t group_half2(const uint4& w, int c) {
  const uint32_t word = (c >> 1) == 0 ? w.x : (c >> 1) == 1 ? w.y : (c >> 1) == 2 ? w.z : w.w;
  return prmt(word, word, (c & 1) ? 0x3232u : 0x1010u);
}

constexpr uint32_t kBias1152x2 = 0x64806480u;  // half2(1152, 1152)

// Biased codes (z + 1152) -> fp16(z * s + b).
__device__ __forceinline__ uint32_t affine_dq(uint32_t biased, uint32_t s2, uint32_t b2) {
  return hfma2_u32(hsub2_u32(biased, kBias1152x2), s2, b2);
}

// Scores of one affine page (log2 units, FP16-path layout: s[0..1] token g,
// s[2..3] token g+8, query rows 2t / 2t+1).  kaddr[kp] = this lane's
// ldmatrix row offset for the chunk pair {2kp, 2kp+1}.
__device__ __forceinline__ void qk_affine(const uint8_t* stage, const uint8_t* meta,
                                          const uint32_t* qa, const uint32_t* kaddr,
                                          float sscale, int valid, int g, float* s) {
  const uint4 ks = lds128(meta, 0);
  const uint4 kb = lds128(meta, 16);
  s[0] = s[1] = s[2] = s[3] = 0.f;
#pragma unroll
  for (int kp = 0; kp < 4; ++kp) {
    uint32_t w[4];  // row g / g+8 of chunk 2kp, row g / g+8 of chunk 2kp+1
    ldsm_x4(stage + kaddr[kp], w[0], w[1], w[2], w[3]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 2 * kp + e;
      const uint32_t s2 = group_half2(ks, c), b2 = group_half2(kb, c);
      const uint32_t wg = w[2 * e], wh = w[2 * e + 1];
      uint32_t a[4];
      a[0] = affine_dq(biased_half2_even(wg), s2, b2);
      a[1] = affine_dq(biased_half2_even(wh), s2, b2);
      a[2] = affine_dq(biased_half2_odd(wg), s2, b2);
      a[3] = affine_dq(biased_half2_odd(wh), s2, b2);
      mma_16816(s, a, qa[2 * c], qa[2 * c + 1]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] *= sscale;
  if (valid < kPage) {
    if (g >= valid) s[0] = s[1] = kNegInf;
    if (g + 8 >= valid) s[2] = s[3] = kNegInf;
  }
}

// PV of one affine page: V tile at stage + 2048 (see pv_int8 for the
// ldmatrix.trans fragment order; m-tile i is dim group i).
__device__ __forceinline__ void pv_affine(WarpState& st, const uint8_t* stage,
                                          const uint8_t* meta, const uint32_t* vaddr,
                                          uint32_t pb0, uint32_t pb1) {
  const uint4 vs = lds128(meta, 32);
  const uint4 vb = lds128(meta, 48);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t r0, r1, r2, r3;  // (tok 0-7, m-tile 2k) (tok 8-15, 2k) (0-7, 2k+1) (8-15, 2k+1)
    ldsm_x4_trans(stage + 2048 + vaddr[k], r0, r1, r2, r3);
    uint32_t s2 = group_half2(vs, 2 * k), b2 = group_half2(vb, 2 * k);
    uint32_t a[4];
    a[0] = affine_dq(biased_half2_even(r0), s2, b2);
    a[1] = affine_dq(biased_half2_odd(r0), s2, b2);
    a[2] = affine_dq(biased_half2_even(r1), s2, b2);
    a[3] = affine_dq(biased_half2_odd(r1), s2, b2);
    mma_16816(st.o + 4 * (2 * k), a, pb0, pb1);
    s2 = group_half2(vs, 2 * k + 1);
    b2 = group_half2(vb, 2 * k + 1);
    a[0] = affine_dq(biased_half2_even(r2), s2, b2);
    a[1] = affine_dq(biased_half2_odd(r2), s2, b2);
    a[2] = affine_dq(biased_half2_even(r3), s2, b2);
    a[3] = affine_dq(biased_half2_odd(r3), s2, b2);
    mma_16816(st.o + 4 * (2 * k + 1), a, pb0, pb1);
  }
}

template <int NP>
__device__ __forceinline__ void pages_affine(WarpState& st, const uint8_t* const* stages,
                                             const uint8_t* const* metas, const uint32_t* qa,
                                             const int* valid, int g, int t, int group,
                                             float sscale, const uint32_t* addr) {
  float s[4 * NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) qk_affine(stages[i], metas[i], qa, addr, sscale, valid[i], g, s + 4 * i);
  uint32_t pb0[NP], pb1[NP];
  float r[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) r[i] = 1.f;
  softmax_pages<NP>(st, s, r, g, t, group, pb0, pb1);
#pragma unroll
  for (int i = 0; i < NP; ++i) pv_affine(st, stages[i], metas[i], addr, pb0[i], pb1[i]);
}

// One pair slot's copies: per page the K and V code tiles (TMA) and the
// page's four 16-byte metadata rows (bulk copies), all on one mbarrier.
__device__ __forceinline__ void issue_pair_affine(const DecodeParams& p, const CUtensorMap* tk,
                                                  const CUtensorMap* tv, uint8_t* dst,
                                                  uint8_t* meta, uint64_t* bar, int n, int id0,
                                                  int id1, int h) {
  const uint64_t pol = l2_evict_first_policy();
  mbar_arrive_expect_tx(bar, n * (4096 + kAffineMetaBytes));
  for (int j = 0; j < n; ++j) {
    const int id = j == 0 ? id0 : id1;
    tma_load_3d_hint(dst + 4096 * j, tk, 0, h, id * kPage, bar, pol);
    tma_load_3d_hint(dst + 4096 * j + 2048, tv, 0, h, id * kPage, bar, pol);
    const int64_t mo = (static_cast<int64_t>(id) * p.hkv + h) * 8;
    uint8_t* m = meta + kAffineMetaBytes * j;
    bulk_load(m, p.seg[0].k_scale + mo, 16, bar);
    bulk_load(m + 16, p.k_bias + mo, 16, bar);
    bulk_load(m + 32, p.seg[0].v_scale + mo, 16, bar);
    bulk_load(m + 48, p.v_bias + mo, 16, bar);
  }
}

// Affine pages of one warp, two at a time, on the pair-slot ring the INT8
// PageGauge loop uses (two slots of two pages, one mbarrier per slot).
__device__ __forceinline__ bool run_warp_pages_affine(
    const DecodeParams& p, const CUtensorMap* tk, const CUtensorMap* tv, WarpState& st,
    uint8_t* ring, uint8_t* meta, uint64_t* bars, uint32_t* qa, int r, int h, int idx_begin,
    int n_pages, bool has_last, int warp, int W, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const SegmentDesc& sd = p.seg[0];
  const int n_w = n_pages > warp ? (n_pages - warp + W - 1) / W : 0;
  if (n_w == 0) return true;
  const int n_pairs = (n_w + 1) >> 1;

  PageWindow win;  // page ids only (the metadata travels with the tiles)
  win.base = 0;
  win.two = n_w > 32;
  load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 0, lane, win.id_a, win.sk_a, win.sv_a);
  win.id_b = 0;
  win.sk_b = win.sv_b = 0.f;
  if (win.two)
    load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, 32, lane, win.id_b, win.sk_b,
                       win.sv_b);

#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if (q < n_pairs) {
      const int u = 2 * q;
      const int n = u + 1 < n_w ? 2 : 1;
      const int id0 = win_id(win, u);
      const int id1 = win_id(win, n == 2 ? u + 1 : u);
      if (lane == 0)
        issue_pair_affine(p, tk, tv, ring + q * 8192, meta + q * 2 * kAffineMetaBytes, bars + q,
                          n, id0, id1, h);
    }
  }

  // ldmatrix row offsets, shared by the K (plain) and V (transposed) reads:
  // lane l addresses row l%8 of matrix l/8; matrices alternate token halves
  // (0-7 / 8-15) and the chunk pair {2k, 2k+1}; chunks are 128B-swizzled.
  uint32_t addr[4];
  {
    const int j = lane >> 3, row = lane & 7;
    const int tok = 8 * (j & 1) + row;
#pragma unroll
    for (int k = 0; k < 4; ++k) addr[k] = tok * 128 + (((2 * k + (j >> 1)) ^ row) << 4);
  }
  pdl_wait_primary();
  int last_valid = kPage;
  if (has_last) {
    const int lv = __ldg(sd.last_len + r);
    last_valid = lv < 1 ? 1 : (lv > kPage ? kPage : lv);
  }
  const bool last_here = has_last && warp + W * (n_w - 1) == n_pages - 1;
  load_q_affine(p, r, h, g, t, qa);

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
    const uint8_t* mt[2] = {meta + (q & 1) * 2 * kAffineMetaBytes,
                            meta + (q & 1) * 2 * kAffineMetaBytes + kAffineMetaBytes};
    int valid[2] = {kPage, kPage};
    if (last_here && q == n_pairs - 1) {
      if (two)
        valid[1] = last_valid;
      else
        valid[0] = last_valid;
    }
    if (two)
      pages_affine<2>(st, stg, mt, qa, valid, g, t, p.group, p.sm_scale_log2, addr);
    else
      pages_affine<1>(st, stg, mt, qa, valid, g, t, p.group, p.sm_scale_log2, addr);
    __syncwarp();
    const int nq = q + 2;
    if (nq < n_pairs) {
      const int nu = 2 * nq;
      const int n = nu + 1 < n_w ? 2 : 1;
      const int id0 = win_id(win, nu);
      const int id1 = win_id(win, n == 2 ? nu + 1 : nu);
      if (lane == 0)
        issue_pair_affine(p, tk, tv, ring + (q & 1) * 8192,
                          meta + (q & 1) * 2 * kAffineMetaBytes, bars + (q & 1), n, id0, id1, h);
    }
    if (win.two && u + 2 - win.base >= 32) {
      win.base += 32;
      win.id_a = win.id_b;
      load_window_set<1>(p, sd, idx_begin, warp, W, n_w, h, win.base + 32, lane, win.id_b,
                         win.sk_b, win.sv_b);
    }
  }
  if (!ok) {
    record_error(p.error_flag, kDevWaitTimeout);
    const int issued_end = q + 2 < n_pairs ? q + 2 : n_pairs;
    for (int v = q; v < issued_end; ++v)
      mbar_wait_bounded(bars + (v & 1), static_cast<uint32_t>(v >> 1) & 1u);
  }
  return ok;
}

}  // namespace pg
