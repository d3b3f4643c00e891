// Bulk quantiser of the "affine_group16" page representation, the
// alternative the reference benchmarks against PageGauge
// (quantize_pages, scripts/benchmark_flashinfer_page_affine_int8.py:234-253),
// restated bit for bit.  Per (page, KV head, group of 16 dims), over the
// group's 16 tokens x 16 dims in FP32:
//   scale = f16(max((max - min) / 255, 2^-20)),   mn = f16(min)
//   u     = clamp(round_half_even((x - mn) / scale), 0, 255)   (IEEE division)
//   code  = u - 128 (int8)
//   bias  = f16(mn + f16(128 * scale))
//   recon = f16(code * scale + bias)   (exact FP32 product, one FP32 add)
// Layouts: values / codes / recon [pages, 16, Hkv, 128]; scale / bias
// [pages, Hkv, 8].  One warp per (page, KV head); lane l owns dims
// 4l..4l+3, so a group is four consecutive lanes.
#pragma once

#include "pg_common.cuh"

namespace pg {

struct AffineQuantParams {
  const __half* values;
  int8_t* codes;
  __half* bias;
  __half* scale;
  __half* recon;  // may be null
  int64_t num_pages;
  int32_t hkv;
};

constexpr int kAffineQuantWarps = 8;

__global__ void __launch_bounds__(kAffineQuantWarps * 32)
    pg_quantize_affine_kernel(const __grid_constant__ AffineQuantParams p) {
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * kAffineQuantWarps + (threadIdx.x >> 5);
  if (wid >= p.num_pages * p.hkv) return;
  const int lane = threadIdx.x & 31;
  const int64_t page = wid / p.hkv;
  const int h = static_cast<int>(wid % p.hkv);
  const int64_t row_stride = static_cast<int64_t>(p.hkv) * kHeadDim;  // one token
  const int64_t base = (page * kPage * p.hkv + h) * kHeadDim + 4 * lane;
  float x[kPage][4];
  float mn = __builtin_huge_valf(), mx = -__builtin_huge_valf();
#pragma unroll
  for (int tok = 0; tok < kPage; ++tok) {
    const uint2 v = *reinterpret_cast<const uint2*>(p.values + base + tok * row_stride);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    x[tok][0] = a.x;
    x[tok][1] = a.y;
    x[tok][2] = b.x;
    x[tok][3] = b.y;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mn = fminf(mn, x[tok][i]);
      mx = fmaxf(mx, x[tok][i]);
    }
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float range_scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 255.f), 0x1p-20f);
  const __half sh = __float2half_rn(range_scale);
  const __half mh = __float2half_rn(mn);
  const float s = __half2float(sh);
  const float m = __half2float(mh);
  const __half b128 = __float2half_rn(128.f * s);
  const __half bh = __float2half_rn(__fadd_rn(m, __half2float(b128)));
  const float bf = __half2float(bh);
#pragma unroll
  for (int tok = 0; tok < kPage; ++tok) {
    int z[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float u = rintf(__fdiv_rn(__fsub_rn(x[tok][i], m), s));
      u = fminf(fmaxf(u, 0.f), 255.f);
      z[i] = static_cast<int>(u) - 128;
    }
    const uint32_t packed = (static_cast<uint32_t>(z[0]) & 0xffu) |
                            ((static_cast<uint32_t>(z[1]) & 0xffu) << 8) |
                            ((static_cast<uint32_t>(z[2]) & 0xffu) << 16) |
                            (static_cast<uint32_t>(z[3]) << 24);
    *reinterpret_cast<uint32_t*>(p.codes + base + tok * row_stride) = packed;
    if (p.recon != nullptr) {
      __half r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        r[i] = __float2half_rn(__fadd_rn(__fmul_rn(static_cast<float>(z[i]), s), bf));
      *reinterpret_cast<uint2*>(p.recon + base + tok * row_stride) =
          *reinterpret_cast<const uint2*>(r);
    }
  }
  if ((lane & 3) == 0) {
    const int64_t mo = (page * p.hkv + h) * 8 + (lane >> 2);
    p.scale[mo] = sh;
    p.bias[mo] = bh;
  }
}

}  // namespace pg
