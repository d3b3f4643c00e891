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
// Layout: CTAs of 256 threads; thread (g, j) = (t / 64, t % 64) owns the
// dimension pair (2j, 2j+1) of one row (a query head, the key or the
// value), so every access is a 4-byte half2 and 64 threads cover one
// coalesced 256-byte FP16 row; for a page close, thread t owns 8
// dimensions (16 bytes) of token t / 16 of the page.  The FP16 comparator
// runs one CTA per (request, KV head); the page-gauge append two (key and
// value), each closing its own page.
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
  // Nonzero: q / k / v are not written by any kernel earlier in the stream
  // (e.g. rows the host wrote before the launch), so the page-gauge append
  // requests them before waiting for the previous kernel.
  int32_t inputs_ready;
  // Served pool layout (the served kernel instantiation only): per batch
  // row the physical token slot in the code pool (page * 16 + token), the
  // token slot in the exact sidecar and the centre row (the request's
  // lease slot); the row's value centre is also copied to center_out
  // [B, Hkv, 128] for the decode's c_V.
  const int32_t* token_slots;
  const int32_t* exact_slots;
  const int32_t* center_rows;
  __half* center_out;
  int64_t num_code_pages, num_exact_pages, num_centers;
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

// A 4-byte word of the new token's q / k / v.  These rows may sit in
// mapped host memory (zero copy, pg_host_device_pointer): ld.cv fetches
// the word over the host link on every call instead of reusing a line an
// earlier launch left in the L2, so each step reads its own inputs.  For
// device memory it is an ordinary L2 load (each word is read once).
__device__ __forceinline__ uint32_t ld_input(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.cv.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// HF rotate-half RoPE for the dims (2j, 2j+1) of one 128-wide head.
__device__ __forceinline__ uint32_t rope_pair(const __half* head, int j,
                                              uint32_t c, uint32_t s) {
  const uint32_t* h32 = reinterpret_cast<const uint32_t*>(head);
  const uint32_t x = ld_input(h32 + j);
  uint32_t partner = ld_input(h32 + ((j + 32) & 63));
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

constexpr int kAppendThreads = 256;

// Loads of one append CTA that do not depend on the position: the token's
// k/v dimension pair (2j, 2j+1) of this KV head and the rotate-half
// partners, issued before the position/RoPE row round trip.
struct AppendInputs {
  uint32_t x, partner;  // k (role 0) or v (role 1) pair, and the k partner
  uint32_t q, qpartner;  // one query head's pair (qh < 0: none)
  int qh;
};

__device__ __forceinline__ uint32_t rope_apply(uint32_t x, uint32_t partner, int j,
                                               uint32_t c, uint32_t s) {
  if (j < 32) partner ^= 0x80008000u;  // -x[d + 64] for d < 64
  return hadd2_rn(hmul2_rn(x, c), hmul2_rn(partner, s));
}

// Thread t = (g, j), g = t / 64: query head h + g*Hkv (+ 4*Hkv ...) and, for
// g = 0 / 1, the key / value pair j of KV head h.
__device__ __forceinline__ AppendInputs load_append_inputs(const AppendParams& p, int r,
                                                           int h, int g, int j) {
  AppendInputs in{};
  in.qh = h + g * p.hkv;
  if (in.qh < p.hq) {
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(
        p.q + r * p.q_stride_b + static_cast<int64_t>(in.qh) * kHeadDim);
    in.q = ld_input(q32 + j);
    in.qpartner = ld_input(q32 + ((j + 32) & 63));
  } else {
    in.qh = -1;
  }
  if (g == 0) {
    const uint32_t* k32 = reinterpret_cast<const uint32_t*>(
        p.k + r * p.k_stride_b + static_cast<int64_t>(h) * kHeadDim);
    in.x = ld_input(k32 + j);
    in.partner = ld_input(k32 + ((j + 32) & 63));
  } else if (g == 1) {
    in.x = ld_input(reinterpret_cast<const uint32_t*>(
                        p.v + r * p.v_stride_b + static_cast<int64_t>(h) * kHeadDim) + j);
  }
  return in;
}

__device__ __forceinline__ void rotate_query_heads(const AppendParams& p, int r, int h, int g,
                                                   int j, const AppendInputs& in, uint32_t c,
                                                   uint32_t s) {
  if (in.qh < 0) return;
  __half* out = p.rotated_q + (static_cast<int64_t>(r) * p.hq) * kHeadDim;
  reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(in.qh) * kHeadDim)[j] =
      rope_apply(in.q, in.qpartner, j, c, s);
  // Groups larger than 4 query heads per KV head: the remaining heads.
  for (int qh = in.qh + 4 * p.hkv; qh < p.hq; qh += 4 * p.hkv) {
    const __half* src = p.q + r * p.q_stride_b + static_cast<int64_t>(qh) * kHeadDim;
    reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(qh) * kHeadDim)[j] =
        rope_pair(src, j, c, s);
  }
}

__global__ void __launch_bounds__(kAppendThreads)
    pg_rope_append_fp16_kernel(const __grid_constant__ AppendParams p) {
  // A dependent decode launch may start streaming completed INT8 pages now
  // (it waits for this grid before reading anything written here); this
  // grid waits for its own predecessor (which produced q, k, v).
  pdl_launch_dependents();
  pdl_wait_primary();
  const int r = blockIdx.x / p.hkv;
  const int h = blockIdx.x % p.hkv;
  const int g = threadIdx.x >> 6, j = threadIdx.x & 63;
  const AppendInputs in = load_append_inputs(p, r, h, g, j);
  int64_t pos;
  const __half *cosr, *sinr;
  if (!resolve_position(p, r, p.exact_pages_per_request * kPage, pos, cosr, sinr)) {
    if (threadIdx.x == 0 && p.device_position != nullptr)
      record_error(p.error_flag, kDevBadPosition);
    return;
  }
  const uint32_t c = reinterpret_cast<const uint32_t*>(cosr)[j];
  const uint32_t s = reinterpret_cast<const uint32_t*>(sinr)[j];
  rotate_query_heads(p, r, h, g, j, in, c, s);
  if (g > 1) return;
  const int64_t page = pos / kPage, token = pos % kPage;
  const int64_t phys = r * p.exact_pages_per_request + page;
  const int64_t dst = ((phys * kPage + token) * p.hkv + h) * kHeadDim;
  if (g == 0)
    reinterpret_cast<uint32_t*>(p.key_pages + dst)[j] = rope_apply(in.x, in.partner, j, c, s);
  else
    reinterpret_cast<uint32_t*>(p.value_pages + dst)[j] = in.x;
}

__device__ __forceinline__ float absmax_half8(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) m = fmaxf(m, absmax2(w[i]));
  return m;
}

// clamp(round_half_away(x / scale)) with the quotient rounded to FP32 as
// an IEEE division would, computed as x * rcp (rcp = 1/scale rounded).
// |x*rcp - x/scale| and |RN(x/scale) - x/scale| are both below 2^-15 for
// |x/scale| <= 128, and the code only changes where the quotient crosses a
// point k + 0.5 (to within one FP32 ulp of |q| + 0.5, <= 2^-16).  So when
// x*rcp lies more than 2^-12 from every k + 0.5 the two quotients give the
// same code; otherwise the exact division decides.
__device__ __forceinline__ int quantize_rcp(float x, float scale, float rcp) {
  const float q = x * rcp;
  const float a = fabsf(q);
  const float f = a - floorf(a);
  if (fabsf(f - 0.5f) <= 0x1p-12f) return quantize_one(x, scale, 0);
  int z = static_cast<int>(floorf(__fadd_rn(a, 0.5f)));
  z = z > 127 ? 127 : z;
  return q < 0.f ? -z : z;
}

// Eight FP16 values -> eight INT8 codes (half away from zero), packed.
__device__ __forceinline__ uint2 quantize_half8(const uint4& v, float scale, float rcp) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hv = *reinterpret_cast<const __half2*>(&w[i]);
    const uint32_t lo = static_cast<uint8_t>(quantize_rcp(__low2float(hv), scale, rcp));
    const uint32_t hi = static_cast<uint8_t>(quantize_rcp(__high2float(hv), scale, rcp));
    out[i >> 1] |= (lo | (hi << 8)) << (16 * (i & 1));
  }
  return make_uint2(out[0], out[1]);
}

// Two CTAs of 256 threads per (request, KV head): role 0 appends and closes
// the key, role 1 the value, and the request's 2*Hkv CTAs share its query
// heads (CTA c = 2h + role rotates heads c, c + 2*Hkv, ...).  Thread
// (g, j) = (t / 64, t % 64): g = 0 rotates (key) and centres its role's
// dimension pair j into the ring slot; g >= 1 rotates pair j of one query
// head.  Page close (token 15): thread t owns 8 consecutive dims (16 B) of
// token t / 16 of the role's page; the 15 older tokens are read from the
// ring as soon as the position is known (alongside the RoPE row), the new
// token comes through shared memory, one CTA reduction gives the abs-max,
// and each thread quantises and writes its 8 codes (one 8-byte store).
// SERVED: pages addressed through the served pool's per-row slots
// (token_slots / exact_slots / center_rows) instead of the request-major
// layout.
template <bool SERVED>
__global__ void __launch_bounds__(kAppendThreads)
    pg_rope_append_page_gauge_kernel(const __grid_constant__ AppendParams p) {
  __shared__ float red[kAppendThreads / 32];
  // A dependent decode launch may start streaming completed INT8 pages now:
  // the page this launch may close is still in the exact window (or the
  // decode was told to request its INT8 tiles only after this grid), and
  // the decode waits for this grid before reading q or the ring.  This grid
  // waits for its own predecessor (which produced q, k, v) before reading
  // anything, unless the caller declared q / k / v ready: then their loads
  // (for host rows, a trip over the host link) overlap the predecessor's
  // tail, and everything else still waits.
  pdl_launch_dependents();
  if (!p.inputs_ready) pdl_wait_primary();
  __shared__ __align__(16) uint32_t newest[kHeadDim / 2];
  const int per_request = 2 * p.hkv;
  const int r = blockIdx.x / per_request;
  const int c = blockIdx.x % per_request;
  const int h = c >> 1, role = c & 1;
  const int g = threadIdx.x >> 6, j = threadIdx.x & 63;
  // Loads that do not depend on the position.
  uint32_t x = 0u, partner = 0u, qx = 0u, qpartner = 0u;
  const int qh = c + (g - 1) * per_request;  // g >= 1: this thread's query head
  if (g == 0) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(
        (role == 0 ? p.k + r * p.k_stride_b : p.v + r * p.v_stride_b) +
        static_cast<int64_t>(h) * kHeadDim);
    x = ld_input(src + j);
    if (role == 0) partner = ld_input(src + ((j + 32) & 63));
  } else if (qh < p.hq) {
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(
        p.q + r * p.q_stride_b + static_cast<int64_t>(qh) * kHeadDim);
    qx = ld_input(q32 + j);
    qpartner = ld_input(q32 + ((j + 32) & 63));
  }
  if (p.inputs_ready) pdl_wait_primary();
  int64_t crow = r;
  if constexpr (SERVED) {
    crow = __ldg(p.center_rows + r);
    if (crow < 0 || crow >= p.num_centers) {
      if (threadIdx.x == 0) record_error(p.error_flag, kDevBadPageId);
      return;
    }
  }
  uint32_t center = 0u;
  if (g == 0) {
    const int64_t cofs = crow * p.center_stride_b + static_cast<int64_t>(h) * kHeadDim;
    center = reinterpret_cast<const uint32_t*>((role == 0 ? p.key_center : p.value_center) +
                                               cofs)[j];
  }
  int64_t pos;
  const __half *cosr, *sinr;
  if (!resolve_position(p, r, p.code_pages_per_request * kPage, pos, cosr, sinr)) {
    if (threadIdx.x == 0 && p.device_position != nullptr)
      record_error(p.error_flag, kDevBadPosition);
    return;
  }
  // Everything the position decides is requested before any store: the
  // RoPE row and, when this token closes the page, the page's 15 older
  // tokens from the ring (stores before them would keep the compiler from
  // issuing those loads early, since it cannot rule out aliasing).
  const int page = static_cast<int>(pos / kPage);
  const int token = static_cast<int>(pos % kPage);
  int64_t ring_page, code_page;
  if constexpr (SERVED) {
    const int32_t ts = __ldg(p.token_slots + r), es = __ldg(p.exact_slots + r);
    if (ts < 0 || es < 0 || (ts & (kPage - 1)) != token || (es & (kPage - 1)) != token ||
        (ts >> 4) >= p.num_code_pages || (es >> 4) >= p.num_exact_pages) {
      if (threadIdx.x == 0) record_error(p.error_flag, kDevBadPageId);
      return;
    }
    ring_page = es >> 4;
    code_page = ts >> 4;
  } else {
    const int sink = static_cast<int>(p.exact_sink_pages);
    const int tail_pages = static_cast<int>(p.exact_pages_per_request) - sink;
    const int local = page < sink ? page : sink + page % tail_pages;
    ring_page = r * p.exact_pages_per_request + local;
    code_page = r * p.code_pages_per_request + page;
  }
  const int64_t row_stride = static_cast<int64_t>(p.hkv) * kHeadDim;  // per token
  __half* ring = (role == 0 ? p.key_pages : p.value_pages) +
                 (ring_page * kPage * p.hkv + h) * kHeadDim;
  // The 16th token closes the page: its INT8 copy is produced now, so it is
  // ready when the page later leaves the exact window.
  const bool close = token == kPage - 1;  // uniform over the CTA
  const int tk = threadIdx.x >> 4, col = (threadIdx.x & 15) * 8;
  uint4 vals = make_uint4(0u, 0u, 0u, 0u);
  if (close && tk < kPage - 1) vals = *reinterpret_cast<const uint4*>(ring + tk * row_stride + col);
  const uint32_t cs = reinterpret_cast<const uint32_t*>(cosr)[j];
  const uint32_t sn = reinterpret_cast<const uint32_t*>(sinr)[j];
  if constexpr (SERVED) {
    if (g == 0 && role == 1)
      reinterpret_cast<uint32_t*>(p.center_out +
                                  (static_cast<int64_t>(r) * p.hkv + h) * kHeadDim)[j] = center;
  }
  if (g >= 1) {
    __half* out = p.rotated_q + static_cast<int64_t>(r) * p.hq * kHeadDim;
    if (qh < p.hq)
      reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(qh) * kHeadDim)[j] =
          rope_apply(qx, qpartner, j, cs, sn);
    // Query heads beyond three per CTA (Hq > 6 * Hkv).
    for (int qo = qh + 3 * per_request; qo < p.hq; qo += 3 * per_request) {
      const __half* src = p.q + r * p.q_stride_b + static_cast<int64_t>(qo) * kHeadDim;
      reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(qo) * kHeadDim)[j] =
          rope_pair(src, j, cs, sn);
    }
  } else {
    const uint32_t val = center_pair(role == 0 ? rope_apply(x, partner, j, cs, sn) : x, center);
    reinterpret_cast<uint32_t*>(ring + token * row_stride)[j] = val;
    if (close) newest[j] = val;
  }
  if (!close) return;
  __syncthreads();
  if (tk == kPage - 1) vals = *reinterpret_cast<const uint4*>(&newest[col / 2]);
  float m = absmax_half8(vals);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kAppendThreads / 32; ++w) m = fmaxf(m, red[w]);
  const __half s_h = __float2half_rn(fmaxf(__fdiv_rn(m, 127.f), 0x1p-20f));
  if (threadIdx.x == 0) (role == 0 ? p.key_scales : p.value_scales)[code_page * p.hkv + h] = s_h;
  const int64_t cbase = (code_page * kPage * p.hkv + h) * kHeadDim + tk * row_stride + col;
  const float sf = __half2float(s_h);
  *reinterpret_cast<uint2*>((role == 0 ? p.key_codes : p.value_codes) + cbase) =
      quantize_half8(vals, sf, __frcp_rn(sf));
}

// Zero the four planes (K/V codes, K/V scales) of the listed pool pages:
// one CTA per listed page; ids outside the pool are skipped and reported.
__global__ void __launch_bounds__(256)
    pg_zero_pool_pages_kernel(int8_t* key_codes, int8_t* value_codes, __half* key_scales,
                              __half* value_scales, int64_t num_pages, int32_t hkv,
                              const int32_t* page_ids, int* error_flag) {
  const int32_t id = __ldg(page_ids + blockIdx.x);
  if (id < 0 || id >= num_pages) {
    if (threadIdx.x == 0) record_error(error_flag, kDevBadPageId);
    return;
  }
  const int64_t chunks = static_cast<int64_t>(kPage) * hkv * kHeadDim / 16;
  uint4* kc = reinterpret_cast<uint4*>(key_codes + static_cast<int64_t>(id) * chunks * 16);
  uint4* vc = reinterpret_cast<uint4*>(value_codes + static_cast<int64_t>(id) * chunks * 16);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int64_t i = threadIdx.x; i < chunks; i += blockDim.x) {
    kc[i] = z;
    vc[i] = z;
  }
  if (threadIdx.x < hkv) {
    key_scales[static_cast<int64_t>(id) * hkv + threadIdx.x] = __float2half_rn(0.f);
    value_scales[static_cast<int64_t>(id) * hkv + threadIdx.x] = __float2half_rn(0.f);
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
  // value == null: key pages only (one tensor to quantise).
  const bool has_v = p.value != nullptr;
  const __half2 kc = reinterpret_cast<const __half2*>(p.key_center + cofs)[j];
  const __half2 vc = has_v ? reinterpret_cast<const __half2*>(p.value_center + cofs)[j]
                           : __floats2half2_rn(0.f, 0.f);
  const int64_t row_stride = static_cast<int64_t>(p.hkv) * kHeadDim;
  const int64_t base = (page * kPage * p.hkv + h) * kHeadDim;
  float2 kf[kPage], vf[kPage];
  float km = 0.f, vm = 0.f;
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    const __half2 kx = reinterpret_cast<const __half2*>(p.key + base + tk * row_stride)[j];
    const __half2 vx = has_v
                           ? reinterpret_cast<const __half2*>(p.value + base + tk * row_stride)[j]
                           : __floats2half2_rn(0.f, 0.f);
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
    if (has_v) p.value_scales[page * p.hkv + h] = vs_h;
  }
  const float ksf = __half2float(ks_h), vsf = __half2float(vs_h);
#pragma unroll
  for (int tk = 0; tk < kPage; ++tk) {
    char2 kz;
    kz.x = quantize_one(kf[tk].x, ksf, p.half_even);
    kz.y = quantize_one(kf[tk].y, ksf, p.half_even);
    reinterpret_cast<char2*>(p.key_codes + base + tk * row_stride)[j] = kz;
    if (has_v) {
      char2 vz;
      vz.x = quantize_one(vf[tk].x, vsf, p.half_even);
      vz.y = quantize_one(vf[tk].y, vsf, p.half_even);
      reinterpret_cast<char2*>(p.value_codes + base + tk * row_stride)[j] = vz;
    }
  }
}

}  // namespace pg
