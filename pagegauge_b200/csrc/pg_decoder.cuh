// Element-wise kernels of the decoder layer around the attention path:
// residual add + RMSNorm, SiLU(gate) * up, and the per-step position
// update.  The arithmetic follows the Mistral decoder layer the reference
// runs (scripts/benchmark_page_gauge_transformer.py:2754-2804 with the
// transformers MistralRMSNorm / SiLU MLP): FP16 storage, FP32 reductions.
//
//   add_rmsnorm:  r = f16(r + d)                      (residual, in place)
//                 y = f16(w * f16(r * rsqrt(mean(r^2) + eps)))
//   silu_mul:     y = f16(f16(g / (1 + exp(-g))) * u)
#pragma once

#include "pg_common.cuh"

namespace pg {

constexpr int kNormThreads = 512;

struct NormParams {
  __half* residual;      // [rows, hidden], updated in place when delta != null
  const __half* delta;   // [rows, hidden] or null
  const __half* weight;  // [hidden]
  __half* out;           // [rows, hidden]
  int64_t residual_stride, delta_stride, out_stride;  // row strides (elements)
  int32_t hidden;        // multiple of 8
  float eps;
};

// One CTA per row; each thread owns 8-element (16-byte) chunks.
__global__ void __launch_bounds__(kNormThreads)
    pg_add_rmsnorm_kernel(const __grid_constant__ NormParams p) {
  __shared__ float part[kNormThreads / 32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const int row = blockIdx.x;
  __half* res = p.residual + row * p.residual_stride;
  const __half* del = p.delta ? p.delta + row * p.delta_stride : nullptr;
  constexpr int kMaxChunks = 4;  // hidden <= 4 * 8 * kNormThreads = 16384
  uint4 x[kMaxChunks];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col >= p.hidden) break;
    x[c] = *reinterpret_cast<const uint4*>(res + col);
    if (del != nullptr) {
      const uint4 d = *reinterpret_cast<const uint4*>(del + col);
      uint32_t* xw = reinterpret_cast<uint32_t*>(&x[c]);
      const uint32_t* dw = reinterpret_cast<const uint32_t*>(&d);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&xw[i]),
                                  *reinterpret_cast<const __half2*>(&dw[i]));
        xw[i] = *reinterpret_cast<const uint32_t*>(&s);
      }
      *reinterpret_cast<uint4*>(res + col) = x[c];
    }
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x[c]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&xw[i]));
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) total += part[w];
  const float inv = rsqrtf(total / static_cast<float>(p.hidden) + p.eps);
  __half* out = p.out + row * p.out_stride;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col >= p.hidden) break;
    const uint4 wv = *reinterpret_cast<const uint4*>(p.weight + col);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x[c]);
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
    uint4 y;
    uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&xw[i]));
      const __half2 n = __floats2half2_rn(f.x * inv, f.y * inv);
      const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&ww[i]), n);
      yw[i] = *reinterpret_cast<const uint32_t*>(&r);
    }
    *reinterpret_cast<uint4*>(out + col) = y;
  }
}

struct SiluMulParams {
  const __half* gate_up;  // [rows, 2F]: gate | up
  __half* out;            // [rows, F]
  int64_t in_stride, out_stride;
  int32_t rows, features;  // F multiple of 8
};

__global__ void __launch_bounds__(256)
    pg_silu_mul_kernel(const __grid_constant__ SiluMulParams p) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int chunks = p.features / 8;
  const int64_t total = static_cast<int64_t>(p.rows) * chunks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / chunks;
    const int col = static_cast<int>(i % chunks) * 8;
    const __half* g = p.gate_up + row * p.in_stride + col;
    const uint4 gv = *reinterpret_cast<const uint4*>(g);
    const uint4 uv = *reinterpret_cast<const uint4*>(g + p.features);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
    uint4 y;
    uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 gf = __half22float2(*reinterpret_cast<const __half2*>(&gw[k]));
      const __half2 s = __floats2half2_rn(gf.x / (1.f + expf(-gf.x)), gf.y / (1.f + expf(-gf.y)));
      const __half2 r = __hmul2(s, *reinterpret_cast<const __half2*>(&uw[k]));
      yw[k] = *reinterpret_cast<const uint32_t*>(&r);
    }
    *reinterpret_cast<uint4*>(p.out + row * p.out_stride + col) = y;
  }
}

// positions[r] += advance; last_len[r] = positions[r] % 16 + 1.
__global__ void pg_step_positions_kernel(int32_t* positions, int32_t* last_len, int32_t batch,
                                         int32_t advance) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= batch) return;
  const int32_t pos = positions[r] + advance;
  positions[r] = pos;
  if (last_len != nullptr) last_len[r] = pos % kPage + 1;
}

// Greedy token per row: the largest logit of a row of FP16 logits and its
// index (ties to the lowest index), one CTA of 1024 threads per row.
constexpr int kArgmaxThreads = 1024;

__global__ void __launch_bounds__(kArgmaxThreads)
    pg_argmax_rows_kernel(const __half* logits, int64_t ld, int32_t cols, int64_t index_offset,
                          float* out_val, int64_t* out_idx) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const __half* row = logits + blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x * 8; c < cols; c += kArgmaxThreads * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(row + c);
    const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __half2float(h[e]);
      if (f > best) {  // columns grow within a thread: the first maximum stays
        best = f;
        bi = c + e;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    // A row of NaN or -inf only: index 0.
    if (bi == 0x7fffffff) bi = 0;
    if (out_val != nullptr) out_val[blockIdx.x] = best;
    out_idx[blockIdx.x] = index_offset + bi;
  }
}

}  // namespace pg
