// Fused RoPE + centred K/V append + completed-page INT8 finalisation, the
// FP16 RoPE+append comparator, and the bulk completed-page quantiser.
//
// Arithmetic contract (bit-exact with the reference extension
// tests/page_gauge_append_extension.cu:148-180, :318-382):
//   rope(x)[d]  = add.rn.f16(mul.rn.f16(x[d], cos[d]),
//                            mul.rn.f16(+-x[d +- 64], sin[d]))   (HF order)
//   centred     = f16_rn(f32(rope_k) - f32(centre))
//   scale       = f16_rn(max(absmax(centred page) / 127 (IEEE), 2^-20))
//   code        = clamp(sign(q) * floor(|q| + 0.5), -127, 127),
//                 q = f32(centred) / f32(scale) (IEEE division)
// The bulk quantiser follows the prefill quantiser instead
// (scripts/benchmark_page_gauge_overheads.py:51-83): fp32 centred values
// that are not rounded to FP16, the same scale rule, and a selectable
// rounding mode (half away from zero, or half to even as torch.round).
//
// Layout: one CTA per (request, KV head), 64 threads; thread j owns the
// dimension pair (2j, 2j+1), so every global access is a 4-byte half2 and a
// 64-thread row is one coalesced 256-byte (FP16) / 128-byte (INT8) line.
#pragma once

#include "pg_common.cuh"

namespace pg {

struct AppendParams {
  const __half* q;
  const __half* k;
  const __half* v;
  int64_t q_stride_b, k_stride_b, v_stride_b;  // batch strides (elements)
  const __half* cos;
  const __half* sin;
  const int32_t* device_position;  // null: use host_position
  int64_t position_stride;          // 0: one position for the batch, 1: per request
  int64_t host_position;
  int64_t rope_row_stride;
  int64_t rope_rows;
  __half* rotated_q;  // [B, Hq, 128] contiguous
  // FP16 cache (comparator) or centred exact ring (page gauge)
  __half* key_pages;
  __half* value_pages;
  // page gauge only
  const __half* key_center;  // [B, Hkv, 128] (or [Hkv,128] with stride 0)
  const __half* value_center;
  int64_t center_stride_b;
  int8_t* key_codes;
  int8_t* value_codes;
  __half* key_scales;
  __half* value_scales;
  int32_t batch, hq, hkv;
  int64_t exact_pages_per_request;  // ring pages per request (page gauge) or
                                    // cache pages per request (FP16)
  int64_t exact_sink_pages;
  int64_t code_pages_per_request;
  int* error_flag;
};

__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hadd2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// HF rotate-half RoPE for the dims (2j, 2j+1) of one 128-wide head.
__device__ __forceinline__ uint32_t rope_pair(const __half* head, int j,
                                              uint32_t c, uint32_t s) {
  const uint32_t* h32 = reinterpret_cast<const uint32_t*>(head);
  const uint32_t x = h32[j];
  uint32_t partner = h32[(j + 32) & 63];
  if (j < 32) partner ^= 0x80008000u;  // -x[d + 64] for d < 64
  return hadd2_rn(hmul2_rn(x, c), hmul2_rn(partner, s));
}

__device__ __forceinline__ uint32_t center_pair(uint32_t x, uint32_t c) {
  const __half2 xh = *reinterpret_cast<const __half2*>(&x);
  const __half2 ch = *reinterpret_cast<const __half2*>(&c);
  const float lo = __fsub_rn(__low2float(xh), __low2float(ch));
  const float hi = __fsub_rn(__high2float(xh), __high2float(ch));
  return pack_half2(lo, hi);
}

__device__ __forceinline__ int round_half_away(float q) {
  return q >= 0.f ? static_cast<int>(floorf(__fadd_rn(q, 0.5f)))
                  : -static_cast<int>(floorf(__fadd_rn(-q, 0.5f)));
}

__device__ __forceinline__ int8_t quantize_one(float x, float scale,
                                               int half_even) {
  const float q = __fdiv_rn(x, scale);
  int z = half_even ? __float2int_rn(q) : round_half_away(q);
  z = z < -127 ? -127 : (z > 127 ? 127 : z);
  return static_cast<int8_t>(z);
}

__device__ __forceinline__ float absmax2(uint32_t v) {
  const __half2 h = *reinterpret_cast<const __half2*>(&v);
  return fmaxf(fabsf(__low2float(h)), fabsf(__high2float(h)));
}

// Reduce a max across the 64-thread CTA.
__device__ __forceinline__ float cta64_max(float v, float* scratch) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  const float r = fmaxf(scratch[0], scratch[1]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ bool resolve_position(const AppendParams& p, int r,
                                                 int64_t capacity_tokens,
                                                 int64_t& pos,
                                                 const __half*& cosr,
                                                 const __half*& sinr) {
  if (p.device_position == nullptr) {
    pos = p.host_position;
    cosr = p.cos;
    sinr = p.sin;
    return pos >= 0 && pos < capacity_tokens;
  }
  pos = __ldg(p.device_position + r * p.position_stride);
  if (pos < 0 || pos >= capacity_tokens || pos >= p.rope_rows) return false;
  cosr = p.cos + pos * p.rope_row_stride;
  sinr = p.sin + pos * p.rope_row_stride;
  return true;
}

// Rotate the query heads h, h + Hkv, ... of request r.
__device__ __forceinline__ void rotate_queries(const AppendParams& p, int r,
                                               int h, int j, uint32_t c,
                                               uint32_t s) {
  for (int qh = h; qh < p.hq; qh += p.hkv) {
    const __half* src = p.q + r * p.q_stride_b + static_cast<int64_t>(qh) * kHeadDim;
    const uint32_t rot = rope_pair(src, j, c, s);
    reinterpret_cast<uint32_t*>(p.rotated_q +
                                (static_cast<int64_t>(r) * p.hq + qh) * kHeadDim)[j] = rot;
  }
}

__global__ void __launch_bounds__(64)
    pg_rope_append_fp16_kernel(const __grid_constant__ AppendParams p) {
  const int r = blockIdx.x / p.hkv;
  const int h = blockIdx.x % p.hkv;
  const int j = threadIdx.x;
  int64_t pos;
  const __half *cosr, *sinr;
  if (!resolve_position(p, r, p.exact_pages_per_request * kPage, pos, cosr, sinr)) {
    if (j == 0 && p.device_position != nullptr)
      record_error(p.error_flag, kDevBadPosition);
    return;
  }
  const uint32_t c = reinterpret_cast<const uint32_t*>(cosr)[j];
  const uint32_t s = reinterpret_cast<const uint32_t*>(sinr)[j];
  rotate_queries(p, r, h, j, c, s);
  const int64_t page = pos / kPage, token = pos % kPage;
  const int64_t phys = r * p.exact_pages_per_request + page;
  const int64_t dst = ((phys * kPage + token) * p.hkv + h) * kHeadDim;
  const __half* kin = p.k + r * p.k_stride_b + static_cast<int64_t>(h) * kHeadDim;
  const __half* vin = p.v + r * p.v_stride_b + static_cast<int64_t>(h) * kHeadDim;
  reinterpret_cast<uint32_t*>(p.key_pages + dst)[j] = rope_pair(kin, j, c, s);
  reinterpret_cast<uint32_t*>(p.value_pages + dst)[j] =
      reinterpret_cast<const uint32_t*>(vin)[j];
}

__global__ void __launch_bounds__(64)
    pg_rope_append_page_gauge_kernel(const __grid_constant__ AppendParams p) {
  __shared__ float red[2];
  const int r = blockIdx.x / p.hkv;
  const int h = blockIdx.x % p.hkv;
  const int j = threadIdx.x;
  int64_t pos;
  const __half *cosr, *sinr;
  if (!resolve_position(p, r, p.code_pages_per_request * kPage, pos, cosr, sinr)) {
    if (j == 0 && p.device_position != nullptr)
      record_error(p.error_flag, kDevBadPosition);
    return;
  }
  const uint32_t c = reinterpret_cast<const uint32_t*>(cosr)[j];
  const uint32_t s = reinterpret_cast<const uint32_t*>(sinr)[j];
  rotate_queries(p, r, h, j, c, s);

  const int64_t page = pos / kPage;
  const int token = static_cast<int>(pos % kPage);
  const int64_t tail_pages = p.exact_pages_per_request - p.exact_sink_pages;
  const int64_t local =
      page < p.exact_sink_pages ? page : p.exact_sink_pages + page % tail_pages;
  const int64_t ring_page = r * p.exact_pages_per_request + local;
  const int64_t code_page = r * p.code_pages_per_request + page;

  const __half* kin = p.k + r * p.k_stride_b + static_cast<int64_t>(h) * kHeadDim;
  const __half* vin = p.v + r * p.v_stride_b + static_cast<int64_t>(h) * kHeadDim;
  const int64_t cofs = r * p.center_stride_b + static_cast<int64_t>(h) * kHeadDim;
  const uint32_t kc = reinterpret_cast<const uint32_t*>(p.key_center + cofs)[j];
  const uint32_t vc = reinterpret_cast<const uint32_t*>(p.value_center + cofs)[j];
  const uint32_t ck = center_pair(rope_pair(kin, j, c, s), kc);
  const uint32_t cv = center_pair(reinterpret_cast<const uint32_t*>(vin)[j], vc);

  const int64_t row_stride = static_cast<int64_t>(p.hkv) * kHeadDim;  // per token
  __half* kring = p.key_pages + (ring_page * kPage * p.hkv + h) * kHeadDim;
  __half* vring = p.value_pages + (ring_page * kPage * p.hkv + h) * kHeadDim;
  reinterpret_cast<uint32_t*>(kring + token * row_stride)[j] = ck;
  reinterpret_cast<uint32_t*>(vring + token * row_stride)[j] = cv;

  // The 16th token closes the page: its INT8 copy is produced now, so it is
  // ready when the page later leaves the exact window.
  if (token != kPage - 1) return;
  uint32_t kv[kPage], vv[kPage];
#pragma unroll
  for (int tk = 0; tk < kPage - 1; ++tk) {
    kv[tk] = reinterpret_cast<const uint32_t*>(kring + tk * row_stride)[j];
    vv[tk] = reinterpret_cast<const uint32_t*>(vring + tk * row_stride)[j];
  }
  kv[kPage - 1] = ck;
  vv[kPage - 1] = cv;
  float km = 0.f, vm = 0.f;
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    km = fmaxf(km, absmax2(kv[tk]));
    vm = fmaxf(vm, absmax2(vv[tk]));
  }
  km = cta64_max(km, red);
  vm = cta64_max(vm, red);
  const __half ks_h = __float2half_rn(fmaxf(__fdiv_rn(km, 127.f), 0x1p-20f));
  const __half vs_h = __float2half_rn(fmaxf(__fdiv_rn(vm, 127.f), 0x1p-20f));
  if (j == 0) {
    p.key_scales[code_page * p.hkv + h] = ks_h;
    p.value_scales[code_page * p.hkv + h] = vs_h;
  }
  const float ksf = __half2float(ks_h), vsf = __half2float(vs_h);
  int8_t* kcode = p.key_codes + (code_page * kPage * p.hkv + h) * kHeadDim;
  int8_t* vcode = p.value_codes + (code_page * kPage * p.hkv + h) * kHeadDim;
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    const __half2 kh = *reinterpret_cast<const __half2*>(&kv[tk]);
    const __half2 vh = *reinterpret_cast<const __half2*>(&vv[tk]);
    char2 kz, vz;
    kz.x = quantize_one(__low2float(kh), ksf, 0);
    kz.y = quantize_one(__high2float(kh), ksf, 0);
    vz.x = quantize_one(__low2float(vh), vsf, 0);
    vz.y = quantize_one(__high2float(vh), vsf, 0);
    reinterpret_cast<char2*>(kcode + tk * row_stride)[j] = kz;
    reinterpret_cast<char2*>(vcode + tk * row_stride)[j] = vz;
  }
}

// ------------------------------------------------ bulk page quantisation
struct QuantizeParams {
  const __half* key;  // [pages, 16, Hkv, 128]
  const __half* value;
  const __half* key_center;  // [num_centers, Hkv, 128]
  const __half* value_center;
  int64_t pages_per_center;  // consecutive pages sharing one centre
  int8_t* key_codes;
  int8_t* value_codes;
  __half* key_scales;  // [pages, Hkv]
  __half* value_scales;
  int64_t num_pages;
  int32_t hkv;
  int32_t half_even;  // 0: half away from zero, 1: half to even
};

// One CTA of 64 threads per (page, KV head); K and V handled together.
__global__ void __launch_bounds__(64)
    pg_quantize_pages_kernel(const __grid_constant__ QuantizeParams p) {
  __shared__ float red[2];
  const int64_t page = blockIdx.x / p.hkv;
  const int h = blockIdx.x % p.hkv;
  const int j = threadIdx.x;
  const int64_t center = p.pages_per_center > 0 ? page / p.pages_per_center : 0;
  const int64_t cofs = (center * p.hkv + h) * kHeadDim;
  const __half2 kc = reinterpret_cast<const __half2*>(p.key_center + cofs)[j];
  const __half2 vc = reinterpret_cast<const __half2*>(p.value_center + cofs)[j];
  const int64_t row_stride = static_cast<int64_t>(p.hkv) * kHeadDim;
  const int64_t base = (page * kPage * p.hkv + h) * kHeadDim;
  float2 kf[kPage], vf[kPage];
  float km = 0.f, vm = 0.f;
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    const __half2 kx = reinterpret_cast<const __half2*>(p.key + base + tk * row_stride)[j];
    const __half2 vx = reinterpret_cast<const __half2*>(p.value + base + tk * row_stride)[j];
    kf[tk].x = __fsub_rn(__low2float(kx), __low2float(kc));
    kf[tk].y = __fsub_rn(__high2float(kx), __high2float(kc));
    vf[tk].x = __fsub_rn(__low2float(vx), __low2float(vc));
    vf[tk].y = __fsub_rn(__high2float(vx), __high2float(vc));
    km = fmaxf(km, fmaxf(fabsf(kf[tk].x), fabsf(kf[tk].y)));
    vm = fmaxf(vm, fmaxf(fabsf(vf[tk].x), fabsf(vf[tk].y)));
  }
  km = cta64_max(km, red);
  vm = cta64_max(vm, red);
  const __half ks_h = __float2half_rn(fmaxf(__fdiv_rn(km, 127.f), 0x1p-20f));
  const __half vs_h = __float2half_rn(fmaxf(__fdiv_rn(vm, 127.f), 0x1p-20f));
  if (j == 0) {
    p.key_scales[page * p.hkv + h] = ks_h;
    p.value_scales[page * p.hkv + h] = vs_h;
  }
  const float ksf = __half2float(ks_h), vsf = __half2float(vs_h);
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    char2 kz, vz;
    kz.x = quantize_one(kf[tk].x, ksf, p.half_even);
    kz.y = quantize_one(kf[tk].y, ksf, p.half_even);
    vz.x = quantize_one(vf[tk].x, vsf, p.half_even);
    vz.y = quantize_one(vf[tk].y, vsf, p.half_even);
    reinterpret_cast<char2*>(p.key_codes + base + tk * row_stride)[j] = kz;
    reinterpret_cast<char2*>(p.value_codes + base + tk * row_stride)[j] = vz;
  }
}

}  // namespace pg
