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

#include "pg_decode_affine.cuh"
#include "pg_decode_core.cuh"
#include "pg_decode_fp16.cuh"
#include "pg_decode_int8.cuh"
#include "pg_merge.cuh"

namespace pg {

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
// representation (kRepGauge or kRepAffine16); WIDE (PageGauge only) is the
// GQA 5-8 form of the INT8 query split.
template <int REP, bool WIDE>
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
      QInt8<WIDE> qi;
      QFragTable* qtab = reinterpret_cast<QFragTable*>(smem + W * kRingBytes + W * kStagesI8 * 8);
      ok = run_warp_pages_int8<WIDE>(p, &tm_k8, &tm_v8, st, ring, bars, qtab, qi, r, h,
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

}  // namespace pg
