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

#include <cooperative_groups.h>

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
};

// Page representations of segment 0 (one kernel instantiation each).
constexpr int kRepGauge = 0;     // one FP16 scale per (page, KV head), centred
constexpr int kRepAffine16 = 1;  // FP16 scale + bias per (page, KV head, 16 dims)

constexpr int kStagesI8 = 4;              // INT8 stages per warp
constexpr int kRingBytes = kStagesI8 * 4096;
constexpr int kMaxWarps = 8;
constexpr int kCoStride = 132;  // padded row of the CTA combine buffer

__host__ __device__ constexpr int decode_smem_bytes(int warps) {
  return warps * kRingBytes + warps * kStagesI8 * 8 + 1024;
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

// Q for the INT8 segment as two int8 parts per row, q ~ sq * (hi + lo/254)
// with sq = max|q_row| / 127 (|error| <= sq/508).  Q is the A operand of
// mma.m16n8k32.s8: rows 0-7 hold the hi parts of the GQA query rows, rows
// 8-15 the lo parts, so one mma yields both partial dot products of a
// query row in the same thread.  a[ks] = {hi dims 32t+8ks+0..3, lo same,
// hi dims 32t+8ks+4..7, lo same} of query row g (the B operand, K, uses
// the identical dimension order).
struct QInt8 {
  uint32_t a[4][4];
  float c;  // sq(row g) / 254 * sm_scale * log2(e)
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

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | (static_cast<uint32_t>(d) << 24);
}

__device__ __forceinline__ int clamp127(int v) { return v < -127 ? -127 : (v > 127 ? 127 : v); }

// Two-part int8 Q for the INT8 segment (thread t owns dims [32t, 32t+32)).
__device__ __forceinline__ void load_q_int8(const DecodeParams& p, int r, int h,
                                            int g, int t, QInt8& qi) {
  float qv[32];
  if (g < p.group) {
    const __half2* q2 = reinterpret_cast<const __half2*>(
        p.q + static_cast<int64_t>(r) * p.q_stride_b +
        static_cast<int64_t>(h * p.group + g) * p.q_stride_h + 32 * t);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 f = __half22float2(q2[i]);
      qv[2 * i] = f.x;
      qv[2 * i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) qv[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(qv[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float sq = amax > 0.f ? amax / 127.f : 1.f;
  const float inv = 1.f / sq;
  const float inv_lo = 254.f / sq;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      int hv[4], lv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = qv[8 * ks + 4 * half + i];
        const int hi = clamp127(__float2int_rn(x * inv));
        const float rem = fmaf(-static_cast<float>(hi), sq, x);
        hv[i] = hi;
        lv[i] = clamp127(__float2int_rn(rem * inv_lo));
      }
      qi.a[ks][2 * half] = pack_s8x4(hv[0], hv[1], hv[2], hv[3]);
      qi.a[ks][2 * half + 1] = pack_s8x4(lv[0], lv[1], lv[2], lv[3]);
    }
  }
  qi.c = sq * (p.sm_scale_log2 / 254.f);
}

__device__ __forceinline__ void mma_s8_16832(int* d, const uint32_t* a,
                                             uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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

// INT8 QK scores of one page for query row g: K tile at stage (16 rows of
// 128 bytes, 128B-swizzled by row) is the B operand straight from shared
// memory (n-tile 0 = tokens 0-7, n-tile 1 = tokens 8-15); the accumulator
// rows g / g+8 carry the hi / lo parts.  s[] = tokens 2t, 2t+1, 8+2t, 9+2t
// in log2 units (masked tokens -inf).
__device__ __forceinline__ void qk_int8(const uint8_t* stage, const QInt8& qi,
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
  const float e = qi.c * sk;
  s[0] = static_cast<float>(c_lo[0] * 254 + c_lo[2]) * e;
  s[1] = static_cast<float>(c_lo[1] * 254 + c_lo[3]) * e;
  s[2] = static_cast<float>(c_hi[0] * 254 + c_hi[2]) * e;
  s[3] = static_cast<float>(c_hi[1] * 254 + c_hi[3]) * e;
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
template <int NP>
__device__ __forceinline__ void pages_int8(WarpState& st,
                                           const uint8_t* const* stages,
                                           const QInt8& qi, const float* sk,
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

__device__ __forceinline__ bool run_warp_pages_int8(
    const DecodeParams& p, const CUtensorMap* tk, const CUtensorMap* tv,
    WarpState& st, uint8_t* ring, uint64_t* bars, QInt8& qi, int r,
    int h, int idx_begin, int n_pages, bool has_last, int warp, int W,
    int lane) {
  const int g = lane >> 2, t = lane & 3;
  const SegmentDesc& sd = p.seg[0];
  const int n_w = n_pages > warp ? (n_pages - warp + W - 1) / W : 0;
  if (n_w == 0) return true;
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
  int last_valid = kPage;
  if (has_last) {
    const int lv = __ldg(sd.last_len + r);
    last_valid = lv < 1 ? 1 : (lv > kPage ? kPage : lv);
  }
  // The warp's last page is the request's last page when it is the item's.
  const bool last_here = has_last && warp + W * (n_w - 1) == n_pages - 1;
  load_q_int8(p, r, h, g, t, qi);

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
      pages_int8<2>(st, stg, qi, sk, rr, valid, g, t, vaddr);
    else
      pages_int8<1>(st, stg, qi, sk, rr, valid, g, t, vaddr);
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

// Merge the optional extra state (lse xl, value read from extra_o), add the
// value centre and store output element (q, d) of head h of request r.
__device__ __forceinline__ void store_final(const DecodeParams& p, int r, int h, int q,
                                            int d, float v, float lv, float xl,
                                            bool write_lse) {
  const int group = p.group;
  const int qh = h * group + q;
  if (p.extra_o != nullptr) {
    const float xo = __half2float(p.extra_o[static_cast<int64_t>(r) * p.extra_stride_b +
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
  if (p.value_center != nullptr)
    v += __half2float(p.value_center[static_cast<int64_t>(r) * p.vc_stride_b + h * kHeadDim + d]);
  p.out[static_cast<int64_t>(r) * p.out_stride_b + static_cast<int64_t>(qh) * p.out_stride_h + d] =
      __float2half_rn(v);
  if (write_lse && p.lse_out != nullptr)
    p.lse_out[static_cast<int64_t>(r) * (p.hkv * group) + qh] = lv;
}

// Last CTA of head h: merge the head's partial states (written by every CTA
// of the head, made visible by the arrival protocol) into the final output.
// Thread -> (query row, 4 dims); partials are folded with an online max.
__device__ __forceinline__ void merge_head(const DecodeParams& p, int r, int h,
                                           const float* xls) {
  const int group = p.group;
  const int rh = r * p.hkv + h;
  const int begin = p.item_off[rh], end = p.item_off[rh + 1];
  for (int slot = threadIdx.x; slot < group * 32; slot += blockDim.x) {
    const int q = slot >> 5, d4 = slot & 31;
    float m = kNegInf, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int U = 8;
    for (int i0 = begin; i0 < end; i0 += U) {
      float l[U];
      float4 v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        l[k] = kNegInf;
        v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i0 + k < end) {
          const int64_t b = static_cast<int64_t>(i0 + k) * group + q;
          l[k] = __ldcg(p.part_lse + b);
          v[k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + b * kHeadDim) + d4);
        }
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        if (l[k] == kNegInf) continue;
        if (l[k] > m) {
          const float sc = fast_exp2(m - l[k]);
          acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
          den *= sc;
          m = l[k];
        }
        const float w = fast_exp2(l[k] - m);
        acc.x += w * v[k].x; acc.y += w * v[k].y; acc.z += w * v[k].z; acc.w += w * v[k].w;
        den += w;
      }
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    const float lv = den > 0.f ? m + fast_log2(den) : kNegInf;
    const float xl = xls[q];
    const int d = 4 * d4;
    store_final(p, r, h, q, d + 0, acc.x * inv, lv, xl, d4 == 0);
    store_final(p, r, h, q, d + 1, acc.y * inv, lv, xl, false);
    store_final(p, r, h, q, d + 2, acc.z * inv, lv, xl, false);
    store_final(p, r, h, q, d + 3, acc.w * inv, lv, xl, false);
  }
}

// Single-launch merge through thread-block clusters.  Every CTA folds its
// warps' states into one normalised state (o, base-2 lse) in its shared
// memory; after a cluster barrier, the cluster's first CTA reads the states
// of its cluster (distributed shared memory) and merges each run of CTAs
// that share a (request, KV head): a run holding all of the head's items
// writes the final output directly, otherwise it stores one partial at the
// run's first item index and the last cluster of the head to arrive (an
// atomic counter per head, re-armed to zero) merges the head's cluster
// partials.  A second cluster barrier keeps every CTA's state alive until
// the first CTA has read it.
// Cluster partials of one head that the finishing CTA weighs through its
// shared-memory table; heads with more take a slower two-pass fold.
constexpr int kClusterMaxParts = 128;

__device__ __noinline__ void cluster_epilogue(const DecodeParams& p, int W, const float* cm,
                                              const float* cl, const float* co, float* xls) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int group = p.group;
  const int total = group * kHeadDim;
  float* st_o = xls + 16;               // [group][128], this CTA's state
  float* st_lse = st_o + 8 * kHeadDim;  // [group]
  float* wts = st_lse + 8;              // [parts][group] merge weights
  float* fin = wts + kClusterMaxParts * 8;  // [group] final lse
  int* s_int = reinterpret_cast<int*>(fin + 8);  // [0] flag, [1..C] run ends
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
        O += co[(w * 8 + q) * kCoStride + d] * e;
      }
    }
    st_o[idx] = L > 0.f ? O / L : 0.f;
    if (d == 0) st_lse[q] = L > 0.f ? M + fast_log2(L) : kNegInf;
  }
  cluster.sync();
  // Turn n states' base-2 lse values (already in wts[j*group + q]) into
  // normalised weights and write the merged lse of each row to fin[q].
  auto weights = [&](int n) {
    __syncthreads();
    if (threadIdx.x < group) {
      const int q = threadIdx.x;
      float M = kNegInf;
      for (int j = 0; j < n; ++j) M = fmaxf(M, wts[j * group + q]);
      float L = 0.f;
      if (M != kNegInf)
        for (int j = 0; j < n; ++j) {
          const float e = wts[j * group + q] == kNegInf ? 0.f : fast_exp2(wts[j * group + q] - M);
          wts[j * group + q] = e;
          L += e;
        }
      else
        for (int j = 0; j < n; ++j) wts[j * group + q] = 0.f;
      const float inv = L > 0.f ? 1.f / L : 0.f;
      for (int j = 0; j < n; ++j) wts[j * group + q] *= inv;
      fin[q] = L > 0.f ? M + fast_log2(L) : kNegInf;
    }
    __syncthreads();
  };
  if (rank == 0) {
    const int base = static_cast<int>(blockIdx.x);
    // Runs of consecutive CTAs of this cluster sharing a (request, head).
    if (threadIdx.x == 0) {
      int k = 0, nr = 0;
      while (k < C && base + k < p.num_items) {
        const DecodeItem it = p.items[base + k];
        int k1 = k + 1;
        while (k1 < C && base + k1 < p.num_items) {
          const DecodeItem nx = p.items[base + k1];
          if (nx.request != it.request || (nx.head_seg & 0xffff) != (it.head_seg & 0xffff)) break;
          ++k1;
        }
        s_int[1 + nr++] = k1;
        k = k1;
      }
      s_int[0] = nr;
    }
    __syncthreads();
    const int nruns = s_int[0];
    int k = 0;
    for (int run = 0; run < nruns; ++run) {
      const int k1 = s_int[1 + run];
      const DecodeItem it = p.items[base + k];
      const int r = it.request, h = it.head_seg & 0xffff;
      const int rh = r * p.hkv + h;
      const int i0 = p.item_off[rh], i1 = p.item_off[rh + 1];
      const bool whole = i0 == base + k && i1 == base + k1;
      const int n = k1 - k;
      for (int e = threadIdx.x; e < n * group; e += blockDim.x)
        wts[e] = cluster.map_shared_rank(st_lse, k + e / group)[e % group];
      if (threadIdx.x < group)
        xls[threadIdx.x] = (whole && p.extra_o != nullptr)
                               ? p.extra_lse[static_cast<int64_t>(r) * (p.hkv * group) +
                                             h * group + threadIdx.x]
                               : kNegInf;
      weights(n);
      // Thread -> 4 consecutive dims of one row: one float4 per state.
      for (int v = threadIdx.x; v < total / 4; v += blockDim.x) {
        const int q = (4 * v) >> 7, d = (4 * v) & 127;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j >= n) break;
          const float w = wts[j * group + q];
          const float4 o = reinterpret_cast<const float4*>(cluster.map_shared_rank(st_o, k + j))[v];
          O.x += w * o.x; O.y += w * o.y; O.z += w * o.z; O.w += w * o.w;
        }
        if (whole) {
          store_final(p, r, h, q, d + 0, O.x, fin[q], xls[q], d == 0);
          store_final(p, r, h, q, d + 1, O.y, fin[q], xls[q], false);
          store_final(p, r, h, q, d + 2, O.z, fin[q], xls[q], false);
          store_final(p, r, h, q, d + 3, O.w, fin[q], xls[q], false);
        } else {
          const int64_t slot = static_cast<int64_t>(base + k) * group + q;
          *reinterpret_cast<float4*>(p.part_o + slot * kHeadDim + d) = O;
          if (d == 0) p.part_lse[slot] = fin[q];
        }
      }
      if (!whole) {
        __threadfence();
        __syncthreads();
        const int first_c = i0 / C, last_c = (i1 - 1) / C;
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(p.sem + rh, 1);
          const int last = prev == last_c - first_c;
          if (last) p.sem[rh] = 0;  // re-armed for the next launch
          s_int[0] = last;
        }
        __syncthreads();
        if (s_int[0]) {
          __threadfence();
          const int parts = last_c - first_c + 1;
          if (threadIdx.x < group)
            xls[threadIdx.x] = p.extra_o != nullptr
                                   ? p.extra_lse[static_cast<int64_t>(r) * (p.hkv * group) +
                                                 h * group + threadIdx.x]
                                   : kNegInf;
          if (parts <= kClusterMaxParts) {
            for (int e = threadIdx.x; e < parts * group; e += blockDim.x) {
              const int c = first_c + e / group;
              wts[e] = __ldcg(p.part_lse + (i0 > c * C ? i0 : c * C) * group + e % group);
            }
            weights(parts);
            // Thread -> 4 consecutive dims of one row; the partials' float4
            // loads go out 16 at a time.
            for (int v = threadIdx.x; v < total / 4; v += blockDim.x) {
              const int q = (4 * v) >> 7, d = (4 * v) & 127;
              float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
              for (int j0 = 0; j0 < parts; j0 += 16) {
                float4 o[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                  const int c = first_c + j0 + u;
                  const int64_t slot = static_cast<int64_t>(i0 > c * C ? i0 : c * C) * group + q;
                  o[u] = j0 + u < parts
                             ? __ldcg(reinterpret_cast<const float4*>(p.part_o + slot * kHeadDim + d))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                  const float w = j0 + u < parts ? wts[(j0 + u) * group + q] : 0.f;
                  O.x += w * o[u].x; O.y += w * o[u].y; O.z += w * o[u].z; O.w += w * o[u].w;
                }
              }
              store_final(p, r, h, q, d + 0, O.x, fin[q], xls[q], d == 0);
              store_final(p, r, h, q, d + 1, O.y, fin[q], xls[q], false);
              store_final(p, r, h, q, d + 2, O.z, fin[q], xls[q], false);
              store_final(p, r, h, q, d + 3, O.w, fin[q], xls[q], false);
            }
          } else {
            // More partials than the weight table holds (very long runs):
            // per row, the maximum and the sum of exp2 over all partials,
            // then each output element folds every partial.
            __syncthreads();
            for (int q = 0; q < group; ++q) {
              float m = kNegInf;
              for (int j = threadIdx.x; j < parts; j += blockDim.x) {
                const int c = first_c + j;
                m = fmaxf(m, __ldcg(p.part_lse + (i0 > c * C ? i0 : c * C) * group + q));
              }
              wts[threadIdx.x] = m;
              __syncthreads();
              if (threadIdx.x == 0) {
                float mm = kNegInf;
                for (int t2 = 0; t2 < static_cast<int>(blockDim.x); ++t2) mm = fmaxf(mm, wts[t2]);
                fin[q] = mm;
              }
              __syncthreads();
              const float M = fin[q];
              float l = 0.f;
              if (M != kNegInf)
                for (int j = threadIdx.x; j < parts; j += blockDim.x) {
                  const int c = first_c + j;
                  const float lj = __ldcg(p.part_lse + (i0 > c * C ? i0 : c * C) * group + q);
                  if (lj != kNegInf) l += fast_exp2(lj - M);
                }
              wts[threadIdx.x] = l;
              __syncthreads();
              if (threadIdx.x == 0) {
                float L = 0.f;
                for (int t2 = 0; t2 < static_cast<int>(blockDim.x); ++t2) L += wts[t2];
                wts[kClusterMaxParts * 8 - 8 + q] = L;  // row sums after the scratch lanes
              }
              __syncthreads();
            }
            for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
              const int q = idx >> 7, d = idx & 127;
              const float M = fin[q], L = wts[kClusterMaxParts * 8 - 8 + q];
              float O = 0.f;
              if (M != kNegInf)
                for (int j = 0; j < parts; ++j) {
                  const int c = first_c + j;
                  const int64_t slot = static_cast<int64_t>(i0 > c * C ? i0 : c * C) * group + q;
                  const float lj = __ldcg(p.part_lse + slot);
                  if (lj != kNegInf) O += fast_exp2(lj - M) * __ldcg(p.part_o + slot * kHeadDim + d);
                }
              store_final(p, r, h, q, d, L > 0.f ? O / L : 0.f,
                          L > 0.f ? M + fast_log2(L) : kNegInf, xls[q], d == 0);
            }
          }
        }
        // s_int[0] (flag) is rewritten by the next run only after a barrier.
      }
      __syncthreads();
      k = k1;
    }
  }
  cluster.sync();
}

// 168 registers per thread at most: three 4-warp CTAs per SM (the host
// planner's slot count assumes it).  REP selects segment 0's page
// representation (kRepGauge or kRepAffine16).
template <int REP>
__global__ void __maxnreg__(168)
    pg_decode_split_kernel(const __grid_constant__ CUtensorMap tm_k8,
                           const __grid_constant__ CUtensorMap tm_v8,
                           const __grid_constant__ CUtensorMap tm_k16,
                           const __grid_constant__ CUtensorMap tm_v16,
                           const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment (128B-swizzled TMA destinations) by pointer
  // arithmetic on the shared array, so loads stay in the shared space.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + W * kRingBytes);
  uint64_t* bars = bars_all + warp * kStagesI8;
  uint8_t* ring = smem + warp * kRingBytes;

  DecodeItem item;
  if (static_cast<int>(blockIdx.x) >= p.num_items) {
    item.request = 0;  // cluster padding: no pages, no output
    item.head_seg = 0;
    item.idx_begin = 0;
    item.count = 0;
  } else if (p.items != nullptr) {
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
  // The dependent grid (the merge, or the next launch) may be scheduled as
  // soon as every CTA of this one has started: its CTAs take SM slots as
  // this grid's CTAs exit and start their own prologue (plan data, first
  // cache tiles) during this grid's drain; they wait for this grid's
  // completion before reading anything it writes.
  pdl_launch_dependents();

  WarpState st;
  st.m0 = st.m1 = kNegInf;
  st.l0 = st.l1 = 0.f;
  st.sref = 1.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) st.o[i] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) st.o1[i] = 0.f;

  bool ok;
  if (seg == 0) {
    if constexpr (REP == kRepGauge) {
      QInt8 qi;
      ok = run_warp_pages_int8(p, &tm_k8, &tm_v8, st, ring, bars, qi, r, h,
                               item.idx_begin, n_pages, has_last, warp, W, lane);
      // Remove the +1152 code bias of the PV operand: O -= 1152 * sum(P'').
      const float sp0 = 1152.f * __shfl_sync(0xffffffffu, st.o1[0], t);
      const float sp1 = 1152.f * __shfl_sync(0xffffffffu, st.o1[1], t);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        st.o[4 * i + 0] -= sp0;
        st.o[4 * i + 1] -= sp1;
        st.o[4 * i + 2] -= sp0;
        st.o[4 * i + 3] -= sp1;
      }
    } else {
      uint8_t* meta = smem + W * kRingBytes + kMaxWarps * kStagesI8 * 8 +
                      warp * kAffineMetaPerWarp;
      uint32_t qa[16];
      ok = run_warp_pages_affine(p, &tm_k8, &tm_v8, st, ring, meta, bars, qa, r, h,
                                 item.idx_begin, n_pages, has_last, warp, W, lane);
    }
  } else {
    uint32_t qf[16];
    ok = run_warp_pages_fp16(p, &tm_k16, &tm_v16, st, ring, bars, qf, r, h,
                           item.idx_begin, n_pages, has_last, warp, W, lane);
  }
  // Warps without pages skipped the wait above; everything below writes.
  pdl_wait_primary();

  // Per-warp totals.  FP16 and affine paths: rows 2t/2t+1, reduce l over
  // the 8 token lanes.  INT8 PageGauge path: row g, reduce l over the 4
  // lanes of the group.
  const bool rowg = REP == kRepGauge && seg == 0;
  if (rowg) {
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, 1);
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, 2);
  } else {
    st.l0 = warp_sum_xor_g(st.l0);
    st.l1 = warp_sum_xor_g(st.l1);
  }
  const float oscale = rowg ? st.sref : 1.f;

  __syncthreads();  // every warp has drained its ring
  const int group = p.group;
  float* cm = reinterpret_cast<float*>(smem);          // [W][8]
  float* cl = cm + kMaxWarps * 8;                      // [W][8]
  float* co = cl + kMaxWarps * 8;                      // [W][8][128]
  const int q0 = 2 * t, q1 = 2 * t + 1;
  if (rowg) {
    if (t == 0) {
      cm[warp * 8 + g] = ok ? st.m0 : kNegInf;
      cl[warp * 8 + g] = ok ? st.l0 : 0.f;
    }
  } else if (g == 0) {
    cm[warp * 8 + q0] = ok ? st.m0 : kNegInf;
    cm[warp * 8 + q1] = ok ? st.m1 : kNegInf;
    cl[warp * 8 + q0] = ok ? st.l0 : 0.f;
    cl[warp * 8 + q1] = ok ? st.l1 : 0.f;
  }
  // Rows of the combine buffer are padded to 132 floats so the float2
  // stores of the 32 lanes fall on distinct bank pairs.
  if (q0 < group) {
    float* c0 = co + (warp * 8 + q0) * kCoStride;
    float* c1 = co + (warp * 8 + q1) * kCoStride;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d0 = seg == 0 ? out_dim<0>(i, g, 0) : out_dim<1>(i, g, 0);
      *reinterpret_cast<float2*>(c0 + d0) =
          make_float2(st.o[4 * i + 0] * oscale, st.o[4 * i + 2] * oscale);
      if (q1 < group)
        *reinterpret_cast<float2*>(c1 + d0) =
            make_float2(st.o[4 * i + 1] * oscale, st.o[4 * i + 3] * oscale);
    }
  }
  __syncthreads();

  // The extra state may alias the outputs (in-place merge): read its lse
  // for every row before any thread writes lse_out.
  float* xls = co + W * 8 * kCoStride;  // [8], inside this CTA's rings
  if (p.final_mode && p.extra_o != nullptr && threadIdx.x < group)
    xls[threadIdx.x] = p.extra_lse[static_cast<int64_t>(r) * (p.hkv * group) + h * group + threadIdx.x];
  __syncthreads();
  if (p.cluster > 1 && !p.final_mode) {
    cluster_epilogue(p, W, cm, cl, co, xls);
    return;
  }
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
        O += co[(w * 8 + q) * kCoStride + d] * e;
      }
    }
    const float on = L > 0.f ? O / L : 0.f;
    const float lse = L > 0.f ? M + fast_log2(L) : kNegInf;
    if (!p.final_mode) {
      const int64_t base = static_cast<int64_t>(blockIdx.x) * group + q;
      p.part_o[base * kHeadDim + d] = on;
      if (d == 0) p.part_lse[base] = lse;
    } else {
      store_final(p, r, h, q, d, on, lse, xls[q], d == 0);
    }
  }
  if (p.final_mode || p.sem == nullptr) return;
  // Fused merge: publish this CTA's partial, count arrivals per head; the
  // last CTA of the head merges.  It also re-arms the counter for the next
  // launch (CUDA-graph replays reuse it).
  __threadfence();
  __syncthreads();
  int* s_last = reinterpret_cast<int*>(xls + 8);
  if (threadIdx.x == 0) {
    const int rh = r * p.hkv + h;
    const int n = p.item_off[rh + 1] - p.item_off[rh];
    const int prev = atomicAdd(p.sem + rh, 1);
    const int last = prev == n - 1;
    if (last) p.sem[rh] = 0;
    *s_last = last;
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  // The extra state may alias out / lse_out: stage its lse first.
  if (threadIdx.x < group)
    xls[threadIdx.x] = p.extra_o != nullptr
                           ? p.extra_lse[static_cast<int64_t>(r) * (p.hkv * group) + h * group + threadIdx.x]
                           : kNegInf;
  __syncthreads();
  merge_head(p, r, h, xls);
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

// One CTA of 256 threads per (request, query head).  Warp w folds the
// partials w, w+8, ... with float4 lanes (4 dims per lane, up to 8 loads in
// flight), then the eight warp states are combined in shared memory and
// thread d < 128 writes output dim d.  The item range is plan data, read
// before waiting on the split kernel.
constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32)
    pg_merge_partials_kernel(const __grid_constant__ MergeParams p) {
  __shared__ float s_m[kMergeWarps], s_den[kMergeWarps];
  __shared__ float4 s_acc[kMergeWarps][32];
  const int hq = p.hkv * p.group;
  const int r = blockIdx.x / hq;
  const int qh = blockIdx.x % hq;
  const int h = qh / p.group, q = qh % p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int begin = p.item_off[r * p.hkv + h];
  const int end = p.item_off[r * p.hkv + h + 1];
  // The next decode launch may start its cache stream now; it waits for this
  // grid before touching anything this grid reads or writes.
  pdl_launch_dependents();
  pdl_wait_primary();
  float m = kNegInf, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int U = 8;
  for (int i0 = begin + warp; i0 < end; i0 += kMergeWarps * U) {
    float l[U];
    float4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int i = i0 + kMergeWarps * k;
      l[k] = kNegInf;
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < end) {
        const int64_t b = static_cast<int64_t>(i) * p.group + q;
        l[k] = __ldcg(p.part_lse + b);
        v[k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + b * kHeadDim) + lane);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      if (l[k] == kNegInf) continue;
      if (l[k] > m) {
        const float sc = fast_exp2(m - l[k]);  // m = -inf -> 0
        acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
        den *= sc;
        m = l[k];
      }
      const float w = fast_exp2(l[k] - m);
      acc.x += w * v[k].x; acc.y += w * v[k].y; acc.z += w * v[k].z; acc.w += w * v[k].w;
      den += w;
    }
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_den[warp] = den;
  }
  s_acc[warp][lane] = acc;
  __syncthreads();
  if (threadIdx.x >= kHeadDim) return;
  const int d = threadIdx.x;
  float M = kNegInf;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) M = fmaxf(M, s_m[w]);
  float D = 0.f, A = 0.f;
  if (M != kNegInf) {
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
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
  // out / lse_out may alias extra_o / extra_lse: all 128 output threads
  // have read them above; sync the four output warps before writing.
  asm volatile("bar.sync 1, 128;" ::: "memory");
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
