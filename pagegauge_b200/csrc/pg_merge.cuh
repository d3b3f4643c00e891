// Cross-CTA merge of the split decode's partial states (one CTA per
// (request, query head)) and merge_state_in_place.
#pragma once

#include "pg_decode_core.cuh"

namespace pg {

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
