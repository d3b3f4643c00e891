// Shared device helpers for the PageGauge B200 kernels (sm_100a only).
//
// Geometry fixed by the PageGauge representation: head_dim 128, 16-token
// pages, NHD page layout [pages, 16, Hkv, 128].  Everything here is plain
// inline PTX for instructions documented in the PTX ISA (mbarrier, bulk
// tensor copies, mma.sync, prmt, ex2.approx) plus small warp utilities.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pg {

constexpr int kHeadDim = 128;
constexpr int kPage = 16;
constexpr float kNegInf = -__builtin_huge_valf();

// Device-side error word.  Kernels never trap: a guard that fires records a
// code here (first writer wins) and the kernel skips the offending work.
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,      // an mbarrier wait exceeded its iteration bound
  kDevBadPosition = 2,      // a device-resident position was out of range
  kDevBadPageId = 3,        // a page-table entry pointed outside the cache
};

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag != nullptr) atomicCAS(flag, 0, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  // Make the initialised barriers visible to the async (TMA) proxy.
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  // The suspend-time hint lets the hardware park the warp until the phase
  // completes (or ~20 us pass) instead of spinning through issue slots.
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return done != 0;
}

// Bounded wait: at most 2^18 suspended polls (seconds), far beyond any
// legitimate TMA latency.  Returns false when the bound is hit; the caller
// records an error and skips the work.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 0; i < (1u << 18); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// ------------------------------------------------------------ wall clock
// The GPU's global nanosecond timer (bounds waits in time, not iterations).
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------- bulk tensor copies
// L2 policy for operands that one launch streams exactly once (cache pages,
// projection weights): their lines are the first to be evicted, so the small
// data every launch re-reads (page tables, scales, queries, activations,
// counters) stays resident in the L2 from one launch to the next.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// 3-D tiled TMA load into this CTA's shared memory, completion signalled on
// an mbarrier by transaction bytes, with an L2 cache policy
// (l2_evict_first_policy for streams).  No multicast: every CTA fetches its
// own tiles from this GPU's memory.
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map,
                                                 int c0, int c1, int c2,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
      "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(
                   reinterpret_cast<uint64_t>(map))
               : "memory");
}

// ------------------------------------------------------------ tensor cores
// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a,
                                          uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------ bit helpers
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Signed INT8 -> FP16 without a conversion instruction: a byte u placed in
// the low mantissa bits of 0x64xx is the half 1024 + u.  With u = z ^ 0x80
// (= z + 128 mod 256) the value is z + 1152 exactly, for every z in
// [-128, 127]; the constant bias is removed after the matrix product.

// Bytes 0 and 2 of w as the biased half2 (z0 + 1152, z2 + 1152): sign-flip,
// mask and exponent in one bitwise select (a single LOP3).
__device__ __forceinline__ uint32_t biased_half2_even(uint32_t w) {
  return ((w ^ 0x64806480u) & 0x00ff00ffu) | (0x64806480u & 0xff00ff00u);
}
// Bytes 1 and 3 of w (shift + LOP3).
__device__ __forceinline__ uint32_t biased_half2_odd(uint32_t w) {
  return biased_half2_even(w >> 8);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_max_xor_g(float v) {
  // Reduce across the 8 lanes sharing lane % 4 (the mma "groupID" axis).
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}

__device__ __forceinline__ float warp_sum_xor_g(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// 16-byte shared-memory load through a plain pointer, so the compiler can
// schedule it freely between the mma/permute instructions while still
// ordering it after the mbarrier wait (which clobbers memory).
__device__ __forceinline__ uint4 lds128(const uint8_t* base, uint32_t offset) {
  return *reinterpret_cast<const uint4*>(base + offset);
}

// Four transposed 8x8 b16 matrices from shared memory; lane l supplies
// the address of row l%8 of matrix l/8 and receives, for matrix j, the
// elements (row 2(l%4), col l/4) and (row 2(l%4)+1, col l/4).
__device__ __forceinline__ void ldsm_x4_trans(const uint8_t* addr, uint32_t& r0,
                                              uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(smem_addr(addr)));
}

// Four 8x8 b16 matrices from shared memory (not transposed); lane l
// supplies the address of row l%8 of matrix l/8 and receives, for matrix j,
// the 32-bit word (l%4) of row l/4.
__device__ __forceinline__ void ldsm_x4(const uint8_t* addr, uint32_t& r0, uint32_t& r1,
                                        uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(addr)));
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Untiled bulk copy global -> this CTA's shared memory, completing on bar
// (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// bulk_load with an L2 cache policy.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch controls (no-ops when launched normally).
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace pg
