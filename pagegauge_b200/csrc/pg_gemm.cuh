// Weight-streaming skinny GEMM for the decoder's projections:
//   Y[b, n] = sum_k X[b, k] * W[n, k]     (b < batch <= 32, W FP16 [n, k])
// with the decoder layer's element-wise step fused into the epilogue.
//
// A decode step reads every weight once and multiplies it by 1..32 token
// rows, so the kernel is an HBM stream of W.  Work is split "stream-K":
// the (output tile, 64-wide k-block) pairs are laid end to end and CTA c
// of G takes blocks [c*T/G, (c+1)*T/G), so every CTA streams the same number
// of bytes whatever the shape.  The weights are stored pre-tiled (one-time
// packing, pg_pack_weight): every (tile, k-block) is a contiguous 8 KB block
// of 64 rows x 64 halves already in the 128-byte-swizzled order ldmatrix
// reads, so a stage's weights are one 8 KB bulk copy (cp.async.bulk) from
// a sequential HBM stream.  A CTA stages its blocks through a 6-deep
// shared-memory ring (activations: tiled TMA, X box 8*NT rows, 128-byte
// swizzle), and its 4 warps run mma.sync m16n8k16 with
// FP32 accumulators (warp w owns W rows 16w..16w+15 of the 64-row tile,
// the batch rows are the n-tiles).  A tile split between CTAs is finished
// by the last of them to arrive (an atomic counter per tile): it sums the
// partial tiles in CTA order (deterministic) and applies the epilogue.
//
// Epilogues (the decoder layer body, transformers Mistral semantics):
//   store     Y = f16(acc)
//   residual  R = f16(R + f16(acc))                   (o_proj, down_proj)
//   silu_mul  Y = f16(f16(silu(f16(acc_gate))) * f16(acc_up)); W rows
//             [0, n/2) are gate rows and [n/2, n) up rows, a 64-row tile
//             holds 32 gate rows and the matching 32 up rows.
// Optional prologue (kernel instantiation NORM): the decoder's RMSNorm of
// the input rows.  Each CTA reduces the rows' sums of squares itself at
// its start, and every activation fragment is normalised in registers
// right after its ldmatrix, f16(w * f16(x * inv_rms)), with no extra
// barrier in the stage loop; this removes the separate norm launch before
// the qkv and gate/up projections.
//
// Programmatic dependent launch: a CTA requests its first weight stages
// before griddepcontrol.wait (weights are never written by a predecessor),
// and the activations only after it.
#pragma once

#include "pg_common.cuh"

namespace pg {

constexpr int kGemmTileRows = 64;  // W rows per output tile
constexpr int kGemmMaxTp = 8;      // ranks of a peer-memory tile exchange
constexpr int kGemmMaxXR = 32;     // activation rows of the widest instantiation

// Exchange buffer of one rank (identical layout on every rank):
//   seq  [cap] int32   exchanges of each output tile completed on this rank
//   recv [2][kGemmMaxTp][cap][64 * kGemmMaxXR] 8-byte (value, tag) words:
//        the tiles by source rank, double-buffered by exchange parity; each
//        word carries one FP32 value (a publishing GEMM: row b, column j at
//        b * 64 + j) or one FP16 pair (pg_tp_publish: columns j, j + 1 at
//        b * 64 + j / 2) with the exchange count as its tag in one store, so
//        a reader knows a value has arrived from the word itself (no
//        separate flag, no fence).
__host__ __device__ constexpr int64_t tp_seq_offset(int) { return 0; }
__host__ __device__ constexpr int64_t tp_recv_offset(int cap) {
  return (static_cast<int64_t>(cap) * 4 + 255) / 256 * 256;
}
__host__ __device__ constexpr int64_t tp_slot_pairs() { return kGemmTileRows * kGemmMaxXR; }
__host__ __device__ constexpr int64_t tp_exchange_bytes(int cap) {
  return tp_recv_offset(cap) + static_cast<int64_t>(2) * kGemmMaxTp * cap * tp_slot_pairs() * 8;
}
constexpr int kGemmBK = 64;        // k per stage: 128-byte rows
// Ring depth: enough weight bytes in flight per SM at the CTAs per SM the
// shared memory allows (3 at 9 KB stages, 2 at 10-12 KB stages).
__host__ __device__ constexpr int gemm_stages(int nt) { return nt == 1 ? 6 : 8; }
constexpr int kGemmWarps = 4;

enum GemmMode { kGemmStore = 0, kGemmResidual = 1, kGemmSiluMul = 2 };

struct GemmParams {
  int32_t n, k, batch, mode;
  int32_t tiles;     // output tiles (mode silu_mul: (n/2)/32, else n/64)
  int32_t kblocks;   // k / 64
  int32_t total;     // tiles * kblocks
  int32_t grid;      // CTAs (<= total; total * grid < 2^31)
  int32_t max_seg;   // tiles one CTA's range can touch
  int32_t half_rows; // mode silu_mul: n / 2 (row offset of the up rows)
  __half* y;
  int64_t ldy;
  __half* residual;
  int64_t ldr;
  float* partials;   // [grid * max_seg][64][8*NT]
  int32_t* counters; // [tiles], zero between launches
  int* error_flag;
  // Tensor-parallel reduction of the finished tiles (world > 1): every
  // rank's exchange buffer as mapped on this rank (peer memory over NVLink,
  // this rank's own included), laid out as pg_tp_exchange_layout describes.
  int32_t tp_world, tp_rank, tp_tiles_cap;
  uint8_t* tp_peers[kGemmMaxTp];
  // Fused RMSNorm prologue (null: none): the GEMM's input is
  // f16(norm_w * f16(x * rsqrt(mean(x^2) + eps))) of the rows of x.
  const __half* norm_w;
  const __half* x;
  int64_t ldx;
  float norm_eps;
};

__host__ __device__ constexpr int gemm_stage_bytes(int nt) {
  return kGemmTileRows * 128 + 8 * nt * 128;
}
__host__ __device__ constexpr int gemm_smem_bytes(int nt) {
  return gemm_stages(nt) * gemm_stage_bytes(nt) + gemm_stages(nt) * 8 + 1024;
}

__device__ __forceinline__ void ldsm_x2(const uint8_t* addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_addr(addr)));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

constexpr int kGemmMaxContrib = 16;  // CTAs sharing one tile (host-checked)

// f16(w * f16(x * inv)) on a half2 (MistralRMSNorm's rounding points).
__device__ __forceinline__ uint32_t rms_scale_h2(uint32_t x, float inv, uint32_t w) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&x));
  const __half2 n = __floats2half2_rn(f.x * inv, f.y * inv);
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&w), n);
  return *reinterpret_cast<const uint32_t*>(&r);
}

// The CTAs whose k-block ranges intersect tile t (ranges are
// [floor(c*T/G), floor((c+1)*T/G))).
__device__ __forceinline__ void gemm_contributors(const GemmParams& p, int t, int& c0, int& c1) {
  c0 = ((t * p.kblocks + 1) * p.grid - 1) / p.total;
  c1 = (((t + 1) * p.kblocks) * p.grid - 1) / p.total;
}

// Request the packed weight block (tile, kb) and expect the whole stage,
// activations included, on the stage's barrier.
template <int NT>
__device__ __forceinline__ void gemm_issue_w(const __half* wp, const GemmParams& p,
                                             uint8_t* stage, uint64_t* bar, int tile, int kb) {
  mbar_arrive_expect_tx(bar, gemm_stage_bytes(NT));
  const __half* src = wp + (static_cast<int64_t>(tile) * p.kblocks + kb) * (kGemmTileRows * kGemmBK);
  bulk_load_hint(stage, src, kGemmTileRows * 128, bar, l2_evict_first_policy());
}

template <int NT>
__device__ __forceinline__ void gemm_issue_x(const CUtensorMap* tx, uint8_t* stage, uint64_t* bar,
                                             int kb) {
  tma_load_2d(stage + kGemmTileRows * 128, tx, kb * kGemmBK, 0, bar);
}

// Epilogue of one finished tile.  `src` gives the FP32 value of (tile row,
// batch row): either this CTA's own accumulators (staged in shared memory)
// or the ordered sum of the contributors' partial tiles.
template <int NT, typename Src>
__device__ __forceinline__ void gemm_epilogue(const GemmParams& p, int tile, Src src) {
  const int rows = p.mode == kGemmSiluMul ? 32 : kGemmTileRows;
  const int count = rows * p.batch;
  for (int e = threadIdx.x; e < count; e += blockDim.x) {
    const int b = e / rows, j = e % rows;
    if (p.mode == kGemmStore) {
      p.y[b * p.ldy + tile * kGemmTileRows + j] = __float2half_rn(src(j, b));
    } else if (p.mode == kGemmResidual) {
      __half* r = p.residual + b * p.ldr + tile * kGemmTileRows + j;
      *r = __hadd(*r, __float2half_rn(src(j, b)));
    } else {
      const float g = __half2float(__float2half_rn(src(j, b)));
      const __half u = __float2half_rn(src(j + 32, b));
      const __half s = __float2half_rn(g / (1.f + expf(-g)));
      p.y[b * p.ldy + tile * 32 + j] = __hmul(s, u);
    }
  }
}

// Tensor-parallel publication of a finished tile: store this rank's FP32
// tile (the batch rows only) into every rank's exchange buffer, each value
// paired with the tile's exchange count in one 8-byte store (plain peer
// stores over NVLink, this rank's own buffer included).  Nothing waits
// here: the ranks' tiles are summed by the kernel that consumes the result
// (pg_tp_reduce_kernel), which waits for the tags, so the GEMM's stream-K
// CTAs never stall on another GPU.  Consecutive exchanges of a tile
// alternate halves of the receive buffer; a rank can be at most one
// exchange ahead of another, because its next exchange's inputs depend on
// this one's reduction on every rank.
// (value, tag) as one 64-bit access, which is single-copy atomic: a reader
// never sees a tag without its value.  The two-element forms move two such
// pairs per instruction (each element still one atomic 64-bit access).
__device__ __forceinline__ void ld_pairs2_relaxed_sys(const uint2* p, uint2& a, uint2& b) {
  unsigned long long x, y;
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p)
               : "memory");
  a = make_uint2(static_cast<uint32_t>(x), static_cast<uint32_t>(x >> 32));
  b = make_uint2(static_cast<uint32_t>(y), static_cast<uint32_t>(y >> 32));
}

__device__ __forceinline__ void st_pairs2_relaxed_sys(uint2* p, float v0, float v1, int32_t tag) {
  const unsigned long long t = static_cast<unsigned long long>(static_cast<uint32_t>(tag)) << 32;
  const unsigned long long x = static_cast<unsigned long long>(__float_as_uint(v0)) | t;
  const unsigned long long y = static_cast<unsigned long long>(__float_as_uint(v1)) | t;
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y)
               : "memory");
}

// Two 8-byte words {v0, tag}, {v1, tag} in one store (v0 / v1: raw bits,
// e.g. an FP16 pair).
__device__ __forceinline__ void st_words2_relaxed_sys(uint2* p, uint32_t v0, uint32_t v1,
                                                      int32_t tag) {
  const unsigned long long t = static_cast<unsigned long long>(static_cast<uint32_t>(tag)) << 32;
  const unsigned long long x = static_cast<unsigned long long>(v0) | t;
  const unsigned long long y = static_cast<unsigned long long>(v1) | t;
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y)
               : "memory");
}

__device__ __forceinline__ uint2 ld_pair_relaxed_sys(const uint2* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return make_uint2(static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32));
}


template <int NT>
__device__ __forceinline__ void gemm_tp_push(const GemmParams& p, int tile, const float* s_tile) {
  constexpr int XR = 8 * NT;
  constexpr int ES = XR + 1;
  __shared__ int s_seq;
  const int cap = p.tp_tiles_cap;
  const int batch = p.batch;
  int32_t* my_seq = reinterpret_cast<int32_t*>(p.tp_peers[p.tp_rank] + tp_seq_offset(cap));
  if (threadIdx.x == 0) s_seq = my_seq[tile];
  __syncthreads();
  const int32_t seq = s_seq + 1;
  const int64_t slot = (static_cast<int64_t>(seq & 1) * kGemmMaxTp + p.tp_rank) * cap + tile;
  // Slot layout [batch row][64 output columns]: a reader's row is contiguous.
  const int n2 = kGemmTileRows / 2 * batch;
  for (int dst = 0; dst < p.tp_world; ++dst) {
    uint2* out = reinterpret_cast<uint2*>(p.tp_peers[dst] + tp_recv_offset(cap)) +
                 slot * tp_slot_pairs();
    for (int i = threadIdx.x; i < n2; i += blockDim.x) {
      const int b = i / (kGemmTileRows / 2), j = 2 * (i - b * (kGemmTileRows / 2));
      st_pairs2_relaxed_sys(out + b * kGemmTileRows + j, s_tile[j * ES + b],
                            s_tile[(j + 1) * ES + b], seq);
    }
  }
  if (threadIdx.x == 0) my_seq[tile] = seq;
  __syncthreads();
}

// Finish this CTA's segment [kb0, kb1) of tile `tile`: the whole tile goes
// straight to the epilogue; a part is written to the CTA's partial slot and
// the last contributor to arrive sums the tile's slots in CTA order.
template <int NT>
__device__ __forceinline__ void gemm_flush(const GemmParams& p, const float (&acc)[NT][4], int tile,
                                           int kb0, int kb1, int seg, float* s_tile, int* s_last,
                                           int* s_seg) {
  constexpr int XR = 8 * NT;
  constexpr int ES = XR + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  if (kb0 == 0 && kb1 == p.kblocks) {
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int row = 16 * warp + g, col = 8 * i + 2 * t;
      s_tile[row * ES + col] = acc[i][0];
      s_tile[row * ES + col + 1] = acc[i][1];
      s_tile[(row + 8) * ES + col] = acc[i][2];
      s_tile[(row + 8) * ES + col + 1] = acc[i][3];
    }
    __syncthreads();
    if (p.tp_world > 1)
      gemm_tp_push<NT>(p, tile, s_tile);
    else
      gemm_epilogue<NT>(p, tile, [&](int j, int b) { return s_tile[j * ES + b]; });
    __syncthreads();
    return;
  }
  const int c = blockIdx.x;
  float* slot = p.partials + (static_cast<int64_t>(c) * p.max_seg + seg) * (kGemmTileRows * XR);
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int row = 16 * warp + g, col = 8 * i + 2 * t;
    *reinterpret_cast<float2*>(slot + row * XR + col) = make_float2(acc[i][0], acc[i][1]);
    *reinterpret_cast<float2*>(slot + (row + 8) * XR + col) = make_float2(acc[i][2], acc[i][3]);
  }
  __threadfence();
  __syncthreads();
  int first, last;
  gemm_contributors(p, tile, first, last);
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + tile, 1);
    const int done = prev == last - first;
    if (done) p.counters[tile] = 0;  // re-armed for the next launch
    *s_last = done;
  }
  // Slot of tile `tile` in each contributor's partials (its segment index).
  if (threadIdx.x <= last - first) {
    const int cc = first + threadIdx.x;
    s_seg[threadIdx.x] = (cc * p.max_seg + tile - (cc * p.total / p.grid) / p.kblocks);
  }
  __syncthreads();
  if (*s_last) {
    __threadfence();
    // Sum the contributors' tiles in CTA order (deterministic): each thread
    // owns float4 chunks of the 64 x XR tile, all contributors' loads of a
    // chunk in flight together, then the sums go through shared memory.
    const int n = last - first + 1;
    constexpr int CH = kGemmTileRows * XR / 4;  // float4 chunks per tile
    for (int ch = threadIdx.x; ch < CH; ch += blockDim.x) {
      float4 v[kGemmMaxContrib];
#pragma unroll
      for (int q = 0; q < kGemmMaxContrib; ++q)
        if (q < n)
          v[q] = __ldcg(reinterpret_cast<const float4*>(
                            p.partials + static_cast<int64_t>(s_seg[q]) * (kGemmTileRows * XR)) +
                        ch);
      float4 acc4 = v[0];
#pragma unroll
      for (int q = 1; q < kGemmMaxContrib; ++q)
        if (q < n) {
          acc4.x += v[q].x;
          acc4.y += v[q].y;
          acc4.z += v[q].z;
          acc4.w += v[q].w;
        }
      const int row = (4 * ch) / XR, col = (4 * ch) % XR;
      s_tile[row * ES + col] = acc4.x;
      s_tile[row * ES + col + 1] = acc4.y;
      s_tile[row * ES + col + 2] = acc4.z;
      s_tile[row * ES + col + 3] = acc4.w;
    }
    __syncthreads();
    if (p.tp_world > 1)
      gemm_tp_push<NT>(p, tile, s_tile);
    else
      gemm_epilogue<NT>(p, tile, [&](int j, int b) { return s_tile[j * ES + b]; });
  }
  __syncthreads();
}

template <int NT, bool NORM>
__global__ void __launch_bounds__(kGemmWarps * 32)
    pg_skinny_gemm_kernel(const __half* __restrict__ w_packed,
                          const __grid_constant__ CUtensorMap tm_x,
                          const __grid_constant__ GemmParams p) {
  constexpr int XR = 8 * NT;            // padded batch rows
  constexpr int SB = gemm_stage_bytes(NT);
  constexpr int kGemmStages = gemm_stages(NT);
  constexpr int ES = XR + 1;            // padded row of the epilogue tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGemmStages * SB);
  __shared__ int s_last;
  __shared__ int s_seg[kGemmMaxContrib];
  __shared__ float s_tile[kGemmTileRows * ES];
  __shared__ float s_inv[XR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int b0 = c * p.total / p.grid, b1 = (c + 1) * p.total / p.grid;
  const int nblk = b1 - b0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) mbar_init(full + s, 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_x);
  }
  __syncthreads();
  // Issue cursor (tile, k-block) of the next block to request.
  int itile = b0 / p.kblocks, ikb = b0 % p.kblocks;
  const int pro = nblk < kGemmStages ? nblk : kGemmStages;
  if (threadIdx.x == 0) {
    int t = itile, k = ikb;
    for (int i = 0; i < pro; ++i) {
      gemm_issue_w<NT>(w_packed, p, smem + i * SB, full + i, t, k);
      if (++k == p.kblocks) k = 0, ++t;
    }
  }
  pdl_launch_dependents();
  pdl_wait_primary();
  if (threadIdx.x == 0) {
    for (int i = 0; i < pro; ++i) {
      gemm_issue_x<NT>(&tm_x, smem + i * SB, full + i, ikb);
      if (++ikb == p.kblocks) ikb = 0, ++itile;
    }
  }
  if constexpr (NORM) {
    // Sum of squares of every input row, all rows at once so that the
    // loads of a pass are independent (one L2 round trip per pass): thread
    // t reads the 16-byte chunks t, t + 128, ... of each row.
    __shared__ float s_red[kGemmWarps][XR];
    const int chunks = p.k / 8;
#pragma unroll 1
    for (int r0 = 0; r0 < XR; r0 += 8) {  // eight rows per pass
      float ss[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) ss[r] = 0.f;
#pragma unroll 2
      for (int ch = threadIdx.x; ch < chunks; ch += kGemmWarps * 32) {
        uint4 v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
          v[r] = r0 + r < p.batch ? reinterpret_cast<const uint4*>(p.x + (r0 + r) * p.ldx)[ch]
                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint32_t w4[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
            ss[r] = fmaf(f.x, f.x, ss[r]);
            ss[r] = fmaf(f.y, f.y, ss[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        float v = ss[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) s_red[warp][r0 + r] = v;
      }
    }
    __syncthreads();
    if (threadIdx.x < XR) {
      const int r = threadIdx.x;
      float total = 0.f;
#pragma unroll
      for (int w = 0; w < kGemmWarps; ++w) total += s_red[w][r];
      s_inv[r] = r < p.batch ? rsqrtf(total / static_cast<float>(p.k) + p.norm_eps) : 0.f;
    }
    __syncthreads();
  }
  // Per n-tile q, the inverse RMS of this lane's batch row 8q + g.
  float inv_g[NT];
#pragma unroll
  for (int q = 0; q < NT; ++q) inv_g[q] = NORM ? s_inv[8 * q + (lane >> 2)] : 0.f;

  // ldmatrix lane addresses (128-byte swizzle: chunk ^ (row & 7)).
  const int mat = lane >> 3, rr = lane & 7;
  const int arow = 16 * warp + rr + 8 * (mat & 1);
  const int achunk = mat >> 1;
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  // Consumer cursor.
  int cur = b0 / p.kblocks, ckb = b0 % p.kblocks;
  int seg = 0;
  int seg_kb0 = ckb;
  bool ok = true;

  int i = 0;
  for (; i < nblk; ++i) {
    if (ckb == p.kblocks) {
      gemm_flush<NT>(p, acc, cur, seg_kb0, p.kblocks, seg, s_tile, &s_last, s_seg);
#pragma unroll
      for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
      ++cur;
      ckb = 0;
      ++seg;
      seg_kb0 = 0;
    }
    const int st = i % kGemmStages;
    const bool waited = mbar_wait_bounded(full + st, static_cast<uint32_t>(i / kGemmStages) & 1u);
    if (!__syncthreads_and(waited)) {
      ok = false;
      break;
    }
    const uint8_t* ws = smem + st * SB;
    const uint8_t* xs = ws + kGemmTileRows * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t a[4];
      ldsm_x4(ws + arow * 128 + (((2 * j + achunk) ^ rr) << 4), a[0], a[1], a[2], a[3]);
      // NORM: this lane's B fragments hold k = 16j + 2t, +1 (x0) and
      // 16j + 8 + 2t, +1 (x1) of batch row 8q + g.
      uint32_t wlo = 0u, whi = 0u;
      if constexpr (NORM) {
        const uint32_t* nw = reinterpret_cast<const uint32_t*>(p.norm_w + ckb * kGemmBK + 16 * j);
        wlo = __ldg(nw + (lane & 3));
        whi = __ldg(nw + 4 + (lane & 3));
      }
#pragma unroll
      for (int q = 0; q < NT; q += 2) {
        if (q + 1 < NT) {
          // Matrices: n-tile q k0-7, k8-15; n-tile q+1 k0-7, k8-15.
          const int xrow = 8 * (q + (mat >> 1)) + rr;
          uint32_t x0, x1, x2, x3;
          ldsm_x4(xs + xrow * 128 + (((2 * j + (mat & 1)) ^ rr) << 4), x0, x1, x2, x3);
          if constexpr (NORM) {
            x0 = rms_scale_h2(x0, inv_g[q], wlo);
            x1 = rms_scale_h2(x1, inv_g[q], whi);
            x2 = rms_scale_h2(x2, inv_g[q + 1], wlo);
            x3 = rms_scale_h2(x3, inv_g[q + 1], whi);
          }
          mma_16816(acc[q], a, x0, x1);
          mma_16816(acc[q + 1], a, x2, x3);
        } else {
          const int xrow = 8 * q + rr;
          uint32_t x0, x1;
          ldsm_x2(xs + xrow * 128 + (((2 * j + (mat & 1)) ^ rr) << 4), x0, x1);
          if constexpr (NORM) {
            x0 = rms_scale_h2(x0, inv_g[q], wlo);
            x1 = rms_scale_h2(x1, inv_g[q], whi);
          }
          mma_16816(acc[q], a, x0, x1);
        }
      }
    }
    ++ckb;
    __syncthreads();  // every warp is done with stage st
    if (threadIdx.x == 0 && i + kGemmStages < nblk) {
      gemm_issue_w<NT>(w_packed, p, smem + st * SB, full + st, itile, ikb);
      gemm_issue_x<NT>(&tm_x, smem + st * SB, full + st, ikb);
      if (++ikb == p.kblocks) ikb = 0, ++itile;
    }
  }
  if (!ok) {
    if (threadIdx.x == 0) record_error(p.error_flag, kDevWaitTimeout);
    // Drain this CTA's copies still in flight before exiting.
    const int end = i + kGemmStages < nblk ? i + kGemmStages : nblk;
    for (int v = i; v < end; ++v)
      mbar_wait_bounded(full + v % kGemmStages, static_cast<uint32_t>(v / kGemmStages) & 1u);
    return;
  }
  gemm_flush<NT>(p, acc, cur, seg_kb0, ckb, seg, s_tile, &s_last, s_seg);
}

// Publication of a partial product computed elsewhere (a library GEMM's
// FP16 output [batch, tiles * 64]): one CTA per output tile stores the
// tile's values into every rank's exchange buffer (this rank's own
// included), then advances the count.  The values are already FP16, so
// each 8-byte word carries an FP16 pair with the tile's exchange count as
// its tag (row b's pairs at b * 64 + j / 2 of the slot): half the bytes of
// the FP32 pairs gemm_tp_push sends, which matters when every rank sends
// every other rank a [32, 4096] partial.  pg_tp_reduce (FP16 payload) then
// sums the same FP16 values in FP32 in rank order.
struct TpPublishParams {
  uint8_t* peers[kGemmMaxTp];
  int32_t world, rank, cap, batch;
  const __half* src;
  int64_t src_stride;
};

constexpr int kTpPublishThreads = 256;

__global__ void __launch_bounds__(kTpPublishThreads)
    pg_tp_publish_kernel(const __grid_constant__ TpPublishParams p) {
  __shared__ int32_t s_seq;
  const int tile = blockIdx.x;
  const int cap = p.cap;
  int32_t* my_seq = reinterpret_cast<int32_t*>(p.peers[p.rank] + tp_seq_offset(cap));
  pdl_launch_dependents();
  pdl_wait_primary();  // the GEMM that wrote src; this rank's previous reduce
  if (threadIdx.x == 0) s_seq = my_seq[tile] + 1;
  __syncthreads();
  const int32_t seq = s_seq;
  const int64_t slot = (static_cast<int64_t>(seq & 1) * kGemmMaxTp + p.rank) * cap + tile;
  // Four columns (two FP16 pairs) per 16-byte store: 16 stores per row.
  const int n4 = kGemmTileRows / 4 * p.batch;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const int b = i / (kGemmTileRows / 4), j = 4 * (i - b * (kGemmTileRows / 4));
    const __half* src = p.src + b * p.src_stride + tile * kGemmTileRows + j;
    const uint32_t v0 = *reinterpret_cast<const uint32_t*>(src);
    const uint32_t v1 = *reinterpret_cast<const uint32_t*>(src + 2);
    for (int dst = 0; dst < p.world; ++dst) {
      uint2* out = reinterpret_cast<uint2*>(p.peers[dst] + tp_recv_offset(cap)) +
                   slot * tp_slot_pairs();
      st_words2_relaxed_sys(out + b * kGemmTileRows + j / 2, v0, v1, seq);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) my_seq[tile] = seq;
}

// Consumer of a tensor-parallel GEMM's published tiles: one CTA of 512
// threads per batch row b.  It waits (bounded) until every rank's tile of
// every output tile has arrived (F16: the FP16-pair words of
// pg_tp_publish; else the FP32 pairs of gemm_tp_push), sums them in rank
// order in FP32 and then
//   residual != null: r = f16(r + f16(sum)); with norm_w, out = RMSNorm(r)
//   residual == null: out = f16(sum)
// (the all-reduce and the decoder's residual add + RMSNorm in one launch).
struct TpReduceParams {
  const uint8_t* exchange;  // this rank's exchange buffer
  int32_t world, cap, tiles;
  __half* residual;
  int64_t residual_stride;
  const __half* norm_w;
  float eps;
  __half* out;
  int64_t out_stride;
  int* error_flag;
};

constexpr int kTpReduceThreads = 512;
constexpr uint64_t kTpWaitNs = 1000000000ull;  // a peer's tiles: wait about a second

template <bool F16>
__global__ void __launch_bounds__(kTpReduceThreads, 1)
    pg_tp_reduce_kernel(const __grid_constant__ TpReduceParams p) {
  __shared__ float part[kTpReduceThreads / 32];
  pdl_launch_dependents();
  pdl_wait_primary();  // the producer GEMM's own pushes and counters
  const uint64_t t0 = globaltimer_ns();
  const int b = blockIdx.x;
  const int cap = p.cap;
  const int32_t* seq = reinterpret_cast<const int32_t*>(p.exchange + tp_seq_offset(cap));
  const uint2* recv = reinterpret_cast<const uint2*>(p.exchange + tp_recv_offset(cap));
  const int n = p.tiles * kGemmTileRows;
  // Thread-owned 8-column chunks, as the add_rmsnorm kernel.
  constexpr int kMaxChunks = 4;  // n <= 4 * 8 * 512
  uint4 x[kMaxChunks];
  float ss = 0.f;
  bool ok = true;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kTpReduceThreads + threadIdx.x) * 8;
    if (col >= n) break;
    const int t = col / kGemmTileRows, j0 = col % kGemmTileRows;
    const int32_t want = __ldcg(seq + t);
    const int par = want & 1;
    float d[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) d[e] = 0.f;
    // Ranks in batches of kSrcBatch: every load of a batch is in flight
    // before the first tag is checked (one memory round trip per batch, not
    // per rank), then only values whose tag is not yet this exchange's
    // count (not arrived) are re-read, for about a second at most.  The
    // sum runs in rank order, identical on every rank.
    constexpr int kSrcBatch = 4;
    constexpr int NP = F16 ? 4 : 8;  // words per 8-column chunk and rank
    for (int s0 = 0; s0 < p.world; s0 += kSrcBatch) {
      uint2 v[kSrcBatch][NP];
      const uint2* rows[kSrcBatch];
#pragma unroll
      for (int k = 0; k < kSrcBatch; ++k) {
        const int src = s0 + k;
        rows[k] = recv + ((static_cast<int64_t>(par) * kGemmMaxTp + src) * cap + t) *
                             tp_slot_pairs() +
                  b * kGemmTileRows + (F16 ? j0 / 2 : j0);  // NP contiguous words
        if (src < p.world) {
#pragma unroll
          for (int e = 0; e < NP; e += 2) ld_pairs2_relaxed_sys(rows[k] + e, v[k][e], v[k][e + 1]);
        }
      }
#pragma unroll
      for (int k = 0; k < kSrcBatch; ++k) {
        if (s0 + k >= p.world) break;
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          for (uint32_t spin = 0; ok && static_cast<int32_t>(v[k][e].y) != want; ++spin) {
            // About a second from the kernel's start (2^26 polls as a backstop).
            if (spin == (1u << 26) ||
                ((spin & 255u) == 255u && globaltimer_ns() - t0 > kTpWaitNs)) {
              ok = false;
              break;
            }
            __nanosleep(32);
            v[k][e] = ld_pair_relaxed_sys(rows[k] + e);
          }
          if constexpr (F16) {
            const uint32_t bits = v[k][e].x;
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&bits));
            d[2 * e] += f.x;
            d[2 * e + 1] += f.y;
          } else {
            d[e] += __uint_as_float(v[k][e].x);
          }
        }
      }
    }
    uint32_t* xw = reinterpret_cast<uint32_t*>(&x[c]);
    if (p.residual != nullptr) {
      __half* res = p.residual + b * p.residual_stride + col;
      const uint4 r = *reinterpret_cast<const uint4*>(res);
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 s2 = __hadd2(*reinterpret_cast<const __half2*>(&rw[e]),
                                   __floats2half2_rn(d[2 * e], d[2 * e + 1]));
        xw[e] = *reinterpret_cast<const uint32_t*>(&s2);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 s2 = __floats2half2_rn(d[2 * e], d[2 * e + 1]);
        xw[e] = *reinterpret_cast<const uint32_t*>(&s2);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  if (!ok) record_error(p.error_flag, kDevWaitTimeout);
  // A row whose tiles did not all arrive in time stores nothing: residual
  // and out keep their contents, so a caller that reads the guard word can
  // repeat the step.
  if (!__syncthreads_and(ok)) return;
  if (p.residual != nullptr) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * kTpReduceThreads + threadIdx.x) * 8;
      if (col >= n) break;
      *reinterpret_cast<uint4*>(p.residual + b * p.residual_stride + col) = x[c];
    }
  }
  float inv = 1.f;
  if (p.norm_w != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kTpReduceThreads / 32; ++w) total += part[w];
    inv = rsqrtf(total / static_cast<float>(n) + p.eps);
  }
  __half* out = p.out + b * p.out_stride;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kTpReduceThreads + threadIdx.x) * 8;
    if (col >= n) break;
    if (p.norm_w == nullptr) {
      *reinterpret_cast<uint4*>(out + col) = x[c];
      continue;
    }
    const uint4 wv = *reinterpret_cast<const uint4*>(p.norm_w + col);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x[c]);
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
    uint4 y;
    uint32_t* yw = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
      const __half2 nrm = __floats2half2_rn(f.x * inv, f.y * inv);
      const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&ww[e]), nrm);
      yw[e] = *reinterpret_cast<const uint32_t*>(&r);
    }
    *reinterpret_cast<uint4*>(out + col) = y;
  }
}

// Weight packing: W [n, k] (row stride ld) -> [tiles][k/64][64][64] with the
// 16-byte chunk c of row r stored at chunk c ^ (r & 7).  Tile t holds rows
// 64t..64t+63, or in silu_mul mode gate rows 32t..32t+31 then the up rows
// n/2 + 32t.. .  One thread per 16-byte chunk.
__global__ void pg_pack_weight_kernel(const __half* __restrict__ w, int64_t ld, int32_t n,
                                      int32_t k, int32_t mode, __half* __restrict__ out) {
  const int kb_count = k / kGemmBK;
  const int64_t chunks = static_cast<int64_t>(n) * (k / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i & 7);
    const int64_t rest = i >> 3;
    const int r = static_cast<int>(rest % kGemmTileRows);
    const int64_t tk = rest / kGemmTileRows;
    const int kb = static_cast<int>(tk % kb_count);
    const int tile = static_cast<int>(tk / kb_count);
    int64_t src_row;
    if (mode == kGemmSiluMul)
      src_row = r < 32 ? tile * 32 + r : n / 2 + tile * 32 + (r - 32);
    else
      src_row = static_cast<int64_t>(tile) * kGemmTileRows + r;
    const uint4 v = *reinterpret_cast<const uint4*>(w + src_row * ld + kb * kGemmBK + c * 8);
    *reinterpret_cast<uint4*>(out + (tk * kGemmTileRows + r) * kGemmBK + ((c ^ (r & 7)) * 8)) = v;
  }
}

}  // namespace pg
