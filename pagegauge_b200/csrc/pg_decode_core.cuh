// Shared pieces of the split-KV decode kernel (pg_decode.cuh): the work
// item and kernel parameter layouts, the per-warp page-id windows, the
// per-warp online-softmax state and the softmax step shared by the FP16 and
// affine paths.
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
  // Fused cross-CTA merge (partial mode): per-(request, head) arrival
  // counters (zero between launches) and the item ranges of each head.  The
  // last CTA of a head merges its partial states into out / lse_out.
  int32_t* sem;
  const int32_t* item_off;
  int* error_flag;
  // > 1: single launch, CTAs grouped in clusters of this many consecutive
  // work items merge their states through distributed shared memory and
  // the last cluster of a head finishes it (no merge kernel).  The grid is
  // padded to whole clusters; CTAs past num_items are empty.
  int32_t cluster;
  // affine_group16 representation (kernel instantiation kRepAffine16):
  // seg[0].k_scale / v_scale are [pages, Hkv, 8] group scales and these the
  // matching group biases.
  const __half* k_bias;
  const __half* v_bias;
  // 1: INT8 tiles only after griddepcontrol.wait (their pages may have been
  // written by a kernel that is still running, e.g. an append that closed
  // a page of a one-page exact ring).
  int32_t int8_after_wait;
};

// Page representations of segment 0 (one kernel instantiation each).
constexpr int kRepGauge = 0;     // one FP16 scale per (page, KV head), centred
constexpr int kRepAffine16 = 1;  // FP16 scale + bias per (page, KV head, 16 dims)

constexpr int kStagesI8 = 4;              // INT8 stages per warp
constexpr int kRingBytes = kStagesI8 * 4096;
constexpr int kMaxWarps = 8;
constexpr int kCoStride = 132;  // padded row of the CTA combine buffer

// The INT8 segment's query, split once per CTA (every warp of a CTA serves
// the same request and KV head): a[lane][4*ks + i] is mma lane `lane`'s
// A-operand register qi.a[ks][i], a2[lane] the wide form's second-MMA
// registers, c[lane] its score factor.
struct QFragTable {
  uint32_t a[32][16];
  uint32_t a2[32][8];
  float c[32];
};
constexpr int kQFragBytes = static_cast<int>(sizeof(QFragTable));

__host__ __device__ constexpr int decode_smem_bytes(int warps) {
  return warps * kRingBytes + warps * kStagesI8 * 8 + kQFragBytes + 1024;
}

// affine_group16: each page also stages its 64 bytes of group metadata
// (k_scale | k_bias | v_scale | v_bias, 8 halves each) after the barriers.
constexpr int kAffineMetaBytes = 64;
constexpr int kAffineMetaPerWarp = kStagesI8 * kAffineMetaBytes;
__host__ __device__ constexpr int decode_smem_bytes_rep(int rep, int warps) {
  return rep == kRepGauge ? decode_smem_bytes(warps)
                          : warps * kRingBytes + kMaxWarps * kStagesI8 * 8 +
                                warps * kAffineMetaPerWarp + 1024;
}

// Output dimension held by accumulator row (m-tile i, row g / g+8).
template <int SEG>
__device__ __forceinline__ int out_dim(int i, int g, int odd) {
  if (SEG == 0) return 16 * i + 2 * g + odd;
  return 64 * (i >> 2) + 8 * g + 2 * (i & 3) + odd;
}

struct WarpState {
  float m0, m1, l0, l1;  // running max / sum for query rows 2t, 2t+1
  float o[32];           // O^T accumulator: 8 m-tiles x (rows g, g+8) x 2 q
  float o1[4];           // "ones" row: sum of the FP16 P'' fed to the PV mma
  float sref;            // reference V scale (INT8 segment)
};

// Q for the INT8 segment as three int8 parts per row,
//   q ~ sq * (hi + lo/254 + lo2/254^2),   sq = max|q_row| / 127,
// |error| <= sq/129032 = max|q_row|/16.4e6 per element (the FP16 input
// itself is only exact to 2^-11 relative).  Two parts (error sq/508) lose
// the small channels of a row that has outlier channels; the third part
// keeps every channel of such a row within FP16 resolution of its largest.
// Q is the A operand of mma.m16n8k32.s8 and a[ks] = {row g dims
// 32t+8ks+0..3, row g+8 same, row g dims 32t+8ks+4..7, row g+8 same}
// (the B operand, K, uses the identical dimension order):
//   GQA group <= 4: rows 0-3 hi, rows 8-11 lo, rows 4-7 lo2 of query rows
//     0-3 (rows 12-15 zero); lane g < 4 adds the lo2 products of lane g+4.
//   GQA group 5-8 (WIDE): rows 0-7 hi, rows 8-15 lo, and a second mma
//     whose rows 0-7 are the lo2 parts (a2 = its non-zero registers).
template <bool WIDE>
struct QInt8 {
  uint32_t a[4][4];
  uint32_t a2[WIDE ? 4 : 1][2];
  float c;  // sq(row g) / 254^2 * sm_scale * log2(e); 0 on lanes holding no row's hi part
};

// A page's scores may exceed the running reference max by this many log2
// units before the output is rescaled (P <= 2^8 stays exact-range in FP16).
constexpr float kRescaleSlack = 8.f;

// Page-id / scale window: lane L of set A holds warp-page base+L, set B
// holds base+32+L.  Shuffles fetch the value of any page in [base, base+64).
struct PageWindow {
  int base;
  bool two;  // more than 32 pages: set B is live
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

// The V/K scales of a window set whose page ids are already loaded (the
// ids gate the first tile copies; the scales are only needed once the
// first tiles have landed, so they are requested after those copies).
__device__ __forceinline__ void load_window_scales(const DecodeParams& p, const SegmentDesc& sd,
                                                   int n_w, int h, int first, int lane, int id,
                                                   float& sk, float& sv) {
  sk = 0.f;
  sv = 0.f;
  if (first + lane < n_w) {
    sk = __half2float(sd.k_scale[static_cast<int64_t>(id) * p.hkv + h]);
    sv = __half2float(sd.v_scale[static_cast<int64_t>(id) * p.hkv + h]);
  }
}

__device__ __forceinline__ int win_id(const PageWindow& w, int u) {
  const int k = u - w.base;
  const int a = __shfl_sync(0xffffffffu, w.id_a, k & 31);
  if (!w.two) return a;
  const int b = __shfl_sync(0xffffffffu, w.id_b, k & 31);
  return k < 32 ? a : b;
}
__device__ __forceinline__ float win_f(const PageWindow& w, float fa, float fb, int k) {
  const float a = __shfl_sync(0xffffffffu, fa, k & 31);
  if (!w.two) return a;
  const float b = __shfl_sync(0xffffffffu, fb, k & 31);
  return k < 32 ? a : b;
}

// Online-softmax update for NP 16-token pages given scaled scores (log2
// units, s[4*i .. 4*i+3] for page i).  The running reference max is only
// raised when some score exceeds it by more than kRescaleSlack, so most
// pages need no cross-lane max and no output rescale.  Returns the packed
// P^T fragments of every page (V scale ratio r[i] folded in).
template <int NP>
__device__ __forceinline__ void softmax_pages(WarpState& st, const float* s,
                                              const float* r, int g, int t,
                                              int group, uint32_t* pb0,
                                              uint32_t* pb1) {
  float lm0 = fmaxf(s[0], s[2]);
  float lm1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int i = 1; i < NP; ++i) {
    lm0 = fmaxf(lm0, fmaxf(s[4 * i + 0], s[4 * i + 2]));
    lm1 = fmaxf(lm1, fmaxf(s[4 * i + 1], s[4 * i + 3]));
  }
  const bool need = (lm0 > st.m0 + kRescaleSlack) || (lm1 > st.m1 + kRescaleSlack);
  if (__any_sync(0xffffffffu, need)) {
    const float mn0 = fmaxf(st.m0, warp_max_xor_g(lm0));
    const float mn1 = fmaxf(st.m1, warp_max_xor_g(lm1));
    const float a0 = mn0 == kNegInf ? 1.f : fast_exp2(st.m0 - mn0);  // -inf -> 0
    const float a1 = mn1 == kNegInf ? 1.f : fast_exp2(st.m1 - mn1);
    st.l0 *= a0;
    st.l1 *= a1;
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
    st.m0 = mn0;
    st.m1 = mn1;
  }
  const float ref0 = st.m0 == kNegInf ? 0.f : st.m0;
  const float ref1 = st.m1 == kNegInf ? 0.f : st.m1;
  const int src0 = 8 * t + (g >> 1);
  const int src1 = src0 + 4;
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const float p0 = fast_exp2(s[4 * i + 0] - ref0);
    const float p1 = fast_exp2(s[4 * i + 1] - ref1);
    const float p2 = fast_exp2(s[4 * i + 2] - ref0);
    const float p3 = fast_exp2(s[4 * i + 3] - ref1);
    st.l0 += p0 + p2;
    st.l1 += p1 + p3;
    const uint32_t h01 = pack_half2(p0 * r[i], p1 * r[i]);
    const uint32_t h23 = pack_half2(p2 * r[i], p3 * r[i]);
    const uint32_t x01 = __shfl_sync(0xffffffffu, h01, src0);
    const uint32_t y01 = __shfl_sync(0xffffffffu, h01, src1);
    const uint32_t x23 = __shfl_sync(0xffffffffu, h23, src0);
    const uint32_t y23 = __shfl_sync(0xffffffffu, h23, src1);
    pb0[i] = g < group ? prmt(x01, y01, sel) : 0u;
    pb1[i] = g < group ? prmt(x23, y23, sel) : 0u;
  }
}

}  // namespace pg
