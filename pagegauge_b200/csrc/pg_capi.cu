// extern "C" entry points of libpagegauge_b200.so: argument validation,
// tensor-map encoding, work planning and kernel launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "pagegauge_b200.h"
#include "pg_affine.cuh"
#include "pg_append.cuh"
#include "pg_decode.cuh"
#include "pg_decoder.cuh"
#include "pg_gemm.cuh"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int32_t cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PG_OK;
  return fail(PG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define PG_REQUIRE(cond, ...)                         \
  do {                                                \
    if (!(cond)) return fail(PG_ERR_INVALID, __VA_ARGS__); \
  } while (0)

// --------------------------------------------------------- device guard
__device__ int g_device_error;

int* device_error_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

// ---------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                   void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault,
                                &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// Page cache [num_pages, 16, Hkv, 128] viewed as rows of 128 bytes:
//   INT8: dims {128 B, Hkv, pages*16}, box {128, 1, 16}
//   FP16: dims {64 halves, 2*Hkv, pages*16}, box {64, 1, 16}
// Both use the 128-byte swizzle so a 16-token tile lands conflict-free.
int32_t make_page_map(CUtensorMap* map, const void* base, int64_t num_pages,
                      int32_t hkv, bool fp16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr)
    return fail(PG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  PG_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0,
             "page cache base must be 16-byte aligned");
  PG_REQUIRE(num_pages > 0 && num_pages * pg::kPage < (int64_t(1) << 31),
             "page cache row count out of range");
  cuuint64_t dims[3];
  cuuint64_t strides[2];
  cuuint32_t box[3];
  const cuuint32_t estr[3] = {1, 1, 1};
  if (!fp16) {
    dims[0] = 128;
    dims[1] = static_cast<cuuint64_t>(hkv);
    dims[2] = static_cast<cuuint64_t>(num_pages) * pg::kPage;
    strides[0] = 128;
    strides[1] = static_cast<cuuint64_t>(hkv) * 128;
    box[0] = 128;
  } else {
    dims[0] = 64;
    dims[1] = static_cast<cuuint64_t>(hkv) * 2;
    dims[2] = static_cast<cuuint64_t>(num_pages) * pg::kPage;
    strides[0] = 128;
    strides[1] = static_cast<cuuint64_t>(hkv) * 256;
    box[0] = 64;
  }
  box[1] = 1;
  box[2] = pg::kPage;
  CUresult r = fn(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                  3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return PG_OK;
}

bool aligned(const void* p, size_t a) {
  return reinterpret_cast<uintptr_t>(p) % a == 0;
}

int32_t ensure_decode_smem() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(PG_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    int32_t rc = cuda_check(
        cudaFuncSetAttribute(pg::pg_decode_split_kernel<pg::kRepGauge, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pg::decode_smem_bytes_rep(pg::kRepGauge, pg::kMaxWarps)),
        "cudaFuncSetAttribute(decode smem)");
    if (rc != PG_OK) return rc;
    rc = cuda_check(
        cudaFuncSetAttribute(pg::pg_decode_split_kernel<pg::kRepGauge, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pg::decode_smem_bytes_rep(pg::kRepGauge, pg::kMaxWarps)),
        "cudaFuncSetAttribute(wide-group decode smem)");
    if (rc != PG_OK) return rc;
    rc = cuda_check(
        cudaFuncSetAttribute(pg::pg_decode_split_kernel<pg::kRepAffine16, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pg::decode_smem_bytes_rep(pg::kRepAffine16, pg::kMaxWarps)),
        "cudaFuncSetAttribute(affine decode smem)");
    if (rc != PG_OK) return rc;
    done[dev] = true;
  }
  return PG_OK;
}

int32_t launch_decode(const pg::DecodeParams& p, const CUtensorMap& k8,
                      const CUtensorMap& v8, const CUtensorMap& k16,
                      const CUtensorMap& v16, int num_ctas, int warps,
                      cudaStream_t stream, int cluster = 1, int rep = pg::kRepGauge) {
  int32_t rc = ensure_decode_smem();
  if (rc != PG_OK) return rc;
  // Programmatic dependent launch: the kernel's prologue (work item, page
  // ids, first INT8 tiles) may overlap the tail of the previous kernel in
  // the stream; it waits for that kernel before reading q or the exact
  // pages and before writing anything.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(num_ctas);
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = pg::decode_smem_bytes_rep(rep, warps);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  if (rep == pg::kRepAffine16)
    return cuda_check(
        cudaLaunchKernelEx(&cfg, pg::pg_decode_split_kernel<pg::kRepAffine16, false>, k8, v8,
                           k16, v16, p),
        "affine decode kernel launch");
  // GQA groups of 5-8 query rows need the second query-split MMA.
  if (p.group > 4)
    return cuda_check(
        cudaLaunchKernelEx(&cfg, pg::pg_decode_split_kernel<pg::kRepGauge, true>, k8, v8, k16,
                           v16, p),
        "decode kernel launch");
  return cuda_check(
      cudaLaunchKernelEx(&cfg, pg::pg_decode_split_kernel<pg::kRepGauge, false>, k8, v8, k16,
                         v16, p),
      "decode kernel launch");
}

// Launch as a programmatic dependent of the previous kernel in the stream:
// the grid may be scheduled while that kernel finishes (hiding the launch
// latency); the kernel itself waits (griddepcontrol.wait) before touching
// anything the predecessor writes.
template <typename... KArgs, typename... Args>
int32_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

// Resident CTAs of the decode kernel per SM at `warps` warps per CTA
// (shared-memory bound: 228 KB per SM, 1 KB reserved per CTA; at most
// 2048 threads and 64 K registers at up to 168 registers per thread).
int pg_ctas_per_sm(int warps) {
  const int by_smem = (228 * 1024) / (pg::decode_smem_bytes(warps) + 1024);
  const int by_threads = 2048 / (warps * 32);
  const int by_regs = 65536 / (warps * 32 * 168);
  return std::max(1, std::min(by_smem, std::min(by_threads, by_regs)));
}

}  // namespace

extern "C" {

const char* pg_last_error(void) { return g_last_error.c_str(); }

int32_t pg_abi_version(void) { return 109; }

int64_t pg_tp_exchange_bytes(int32_t tiles_cap) {
  return tiles_cap > 0 ? pg::tp_exchange_bytes(tiles_cap) : -1;
}

int32_t pg_tp_exchange_create(int32_t tiles_cap, void** buffer_out, void* ipc_handle_out) {
  PG_REQUIRE(tiles_cap > 0 && tiles_cap <= (1 << 16), "tile capacity out of range");
  PG_REQUIRE(buffer_out != nullptr && ipc_handle_out != nullptr, "null pointer");
  void* ptr = nullptr;
  const size_t bytes = static_cast<size_t>(pg::tp_exchange_bytes(tiles_cap));
  int32_t rc = cuda_check(cudaMalloc(&ptr, bytes), "cudaMalloc(exchange buffer)");
  if (rc != PG_OK) return rc;
  rc = cuda_check(cudaMemset(ptr, 0, bytes), "cudaMemset(exchange buffer)");
  if (rc == PG_OK) {
    cudaIpcMemHandle_t h;
    rc = cuda_check(cudaIpcGetMemHandle(&h, ptr), "cudaIpcGetMemHandle");
    if (rc == PG_OK) std::memcpy(ipc_handle_out, &h, sizeof(h));
  }
  if (rc != PG_OK) {
    cudaFree(ptr);
    return rc;
  }
  *buffer_out = ptr;
  return PG_OK;
}

int32_t pg_tp_exchange_open(const void* ipc_handle, void** buffer_out) {
  PG_REQUIRE(ipc_handle != nullptr && buffer_out != nullptr, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* ptr = nullptr;
  int32_t rc = cuda_check(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                          "cudaIpcOpenMemHandle");
  if (rc != PG_OK) return rc;
  *buffer_out = ptr;
  return PG_OK;
}

int32_t pg_tp_exchange_close(void* peer_buffer) {
  PG_REQUIRE(peer_buffer != nullptr, "null pointer");
  return cuda_check(cudaIpcCloseMemHandle(peer_buffer), "cudaIpcCloseMemHandle");
}

int32_t pg_tp_exchange_destroy(void* buffer) {
  PG_REQUIRE(buffer != nullptr, "null pointer");
  return cuda_check(cudaFree(buffer), "cudaFree(exchange buffer)");
}

int32_t pg_host_device_pointer(const void* host, void** device_out) {
  PG_REQUIRE(host != nullptr && device_out != nullptr, "null pointer");
  void* d = nullptr;
  int32_t rc = cuda_check(cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0),
                          "cudaHostGetDevicePointer (the buffer must be page-locked and mapped)");
  if (rc != PG_OK) return rc;
  *device_out = d;
  return PG_OK;
}

int32_t pg_struct_sizes(int64_t* out, int32_t n) {
  PG_REQUIRE(out != nullptr && n >= 5, "need room for 5 sizes");
  out[0] = sizeof(pg_decode_args);
  out[1] = sizeof(pg_gemm_args);
  out[2] = sizeof(pg_segment);
  out[3] = sizeof(pg_plan_info);
  out[4] = sizeof(pg_decode_item);
  return PG_OK;
}

int32_t pg_read_device_error(int32_t* code_out) {
  int* p = device_error_ptr();
  if (p == nullptr) return fail(PG_ERR_CUDA, "device error word unavailable");
  int v = 0;
  int32_t rc = cuda_check(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost),
                          "read device error");
  if (rc != PG_OK) return rc;
  int zero = 0;
  rc = cuda_check(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice),
                  "clear device error");
  if (code_out) *code_out = v;
  return rc;
}

// ------------------------------------------------------------------ append
static int32_t append_fp16_impl(const void* query, const void* key,
                                const void* value, const void* cosine,
                                const void* sine, void* rotated_query,
                                void* key_pages, void* value_pages,
                                int64_t query_batch_stride,
                                int64_t key_batch_stride,
                                int64_t value_batch_stride, int32_t batch,
                                int32_t query_heads, int32_t kv_heads,
                                int64_t num_pages, int64_t position,
                                const int32_t* device_position,
                                int64_t position_stride,
                                int64_t rope_row_stride, int64_t rope_rows,
                                void* stream) {
  PG_REQUIRE(batch > 0, "Q/K/V batch sizes must match and be positive");
  PG_REQUIRE(query_heads > 0 && kv_heads > 0, "head counts must be positive");
  if (device_position == nullptr) {
    PG_REQUIRE(position >= 0, "position must be non-negative");
    PG_REQUIRE(position / pg::kPage < num_pages,
               "position exceeds the allocated FP16 cache");
  } else {
    PG_REQUIRE(rope_rows > 0, "dynamic RoPE tables must be matching [positions,128] tensors");
  }
  PG_REQUIRE(num_pages % batch == 0, "FP16 cache pages must divide evenly across requests");
  const int64_t ppr = num_pages / batch;
  if (device_position == nullptr)
    PG_REQUIRE(position / pg::kPage < ppr,
               "position exceeds the per-request FP16 cache capacity");
  PG_REQUIRE(aligned(query, 4) && aligned(key, 4) && aligned(value, 4) &&
                 aligned(cosine, 4) && aligned(sine, 4) && aligned(key_pages, 4) &&
                 aligned(value_pages, 4) && aligned(rotated_query, 4),
             "tensors must be 4-byte aligned");
  PG_REQUIRE(query_batch_stride % 2 == 0 && key_batch_stride % 2 == 0 &&
                 value_batch_stride % 2 == 0 && rope_row_stride % 2 == 0,
             "batch strides must be even");
  pg::AppendParams p{};
  p.q = static_cast<const __half*>(query);
  p.k = static_cast<const __half*>(key);
  p.v = static_cast<const __half*>(value);
  p.q_stride_b = query_batch_stride;
  p.k_stride_b = key_batch_stride;
  p.v_stride_b = value_batch_stride;
  p.cos = static_cast<const __half*>(cosine);
  p.sin = static_cast<const __half*>(sine);
  p.device_position = device_position;
  p.position_stride = position_stride;
  p.host_position = position;
  p.rope_row_stride = rope_row_stride;
  p.rope_rows = rope_rows;
  p.rotated_q = static_cast<__half*>(rotated_query);
  p.key_pages = static_cast<__half*>(key_pages);
  p.value_pages = static_cast<__half*>(value_pages);
  p.batch = batch;
  p.hq = query_heads;
  p.hkv = kv_heads;
  p.exact_pages_per_request = ppr;
  p.error_flag = device_error_ptr();
  return launch_pdl(pg::pg_rope_append_fp16_kernel, dim3(batch * kv_heads),
                    dim3(pg::kAppendThreads), 0, static_cast<cudaStream_t>(stream),
                    "rope_append_fp16 launch", p);
}

int32_t pg_rope_append_fp16(const void* query, const void* key,
                            const void* value, const void* cosine,
                            const void* sine, void* rotated_query,
                            void* key_pages, void* value_pages,
                            int64_t query_batch_stride,
                            int64_t key_batch_stride,
                            int64_t value_batch_stride, int32_t batch,
                            int32_t query_heads, int32_t kv_heads,
                            int64_t num_pages, int64_t position,
                            const int32_t* device_position,
                            int64_t rope_row_stride, int64_t rope_rows,
                            void* stream) {
  return append_fp16_impl(query, key, value, cosine, sine, rotated_query, key_pages,
                          value_pages, query_batch_stride, key_batch_stride,
                          value_batch_stride, batch, query_heads, kv_heads, num_pages,
                          position, device_position, 0, rope_row_stride, rope_rows, stream);
}

int32_t pg_rope_append_fp16_batched(const void* query, const void* key,
                                    const void* value, const void* cosine,
                                    const void* sine, void* rotated_query,
                                    void* key_pages, void* value_pages,
                                    int64_t query_batch_stride,
                                    int64_t key_batch_stride,
                                    int64_t value_batch_stride, int32_t batch,
                                    int32_t query_heads, int32_t kv_heads,
                                    int64_t num_pages, const int32_t* positions,
                                    int64_t rope_row_stride, int64_t rope_rows,
                                    void* stream) {
  PG_REQUIRE(positions != nullptr, "per-request positions must be a device int32 [B] tensor");
  return append_fp16_impl(query, key, value, cosine, sine, rotated_query, key_pages,
                          value_pages, query_batch_stride, key_batch_stride,
                          value_batch_stride, batch, query_heads, kv_heads, num_pages, 0,
                          positions, 1, rope_row_stride, rope_rows, stream);
}

static int32_t append_page_gauge_impl(
    const void* query, const void* key, const void* value,
    const void* cosine, const void* sine, const void* key_center,
    const void* value_center, void* rotated_query, void* exact_key_pages,
    void* exact_value_pages, void* key_codes, void* value_codes,
    void* key_scales, void* value_scales, int64_t query_batch_stride,
    int64_t key_batch_stride, int64_t value_batch_stride,
    int64_t center_batch_stride, int32_t batch, int32_t query_heads,
    int32_t kv_heads, int64_t exact_pages, int64_t code_pages,
    int64_t exact_sink_pages, int64_t position,
    const int32_t* device_position, int64_t position_stride,
    int64_t rope_row_stride, int64_t rope_rows, void* stream, int32_t inputs_ready = 0) {
  PG_REQUIRE(batch > 0, "Q/K/V batch sizes must match and be positive");
  PG_REQUIRE(query_heads > 0 && kv_heads > 0, "head counts must be positive");
  if (device_position == nullptr) {
    PG_REQUIRE(position >= 0, "position must be non-negative");
  } else {
    PG_REQUIRE(rope_rows > 0, "dynamic RoPE tables must be matching [positions,128] tensors");
  }
  PG_REQUIRE(exact_pages > 0 && exact_pages % batch == 0 && code_pages % batch == 0,
             "PageGauge pages must be positive and divide evenly across requests");
  const int64_t exact_ppr = exact_pages / batch;
  PG_REQUIRE(exact_sink_pages >= 0, "exact prefix page count must be nonnegative");
  PG_REQUIRE(exact_ppr > exact_sink_pages,
             "exact cache must retain at least one tail-ring page");
  const int64_t code_ppr = code_pages / batch;
  PG_REQUIRE(exact_sink_pages < code_ppr,
             "exact prefix exceeds the logical cache capacity");
  if (device_position == nullptr)
    PG_REQUIRE(position / pg::kPage < code_ppr,
               "position exceeds the per-request PageGauge cache capacity");
  PG_REQUIRE(aligned(query, 4) && aligned(key, 4) && aligned(value, 4) &&
                 aligned(cosine, 4) && aligned(sine, 4) && aligned(key_center, 4) &&
                 aligned(value_center, 4) && aligned(exact_key_pages, 4) &&
                 aligned(exact_value_pages, 4) && aligned(key_codes, 2) &&
                 aligned(value_codes, 2) && aligned(rotated_query, 4),
             "tensors must be 4-byte aligned");
  // The page close reads the ring page in 16-byte rows and writes codes in
  // 8-byte rows.
  PG_REQUIRE(aligned(exact_key_pages, 16) && aligned(exact_value_pages, 16) &&
                 aligned(key_codes, 8) && aligned(value_codes, 8),
             "exact pages must be 16-byte and INT8 codes 8-byte aligned");
  PG_REQUIRE(query_batch_stride % 2 == 0 && key_batch_stride % 2 == 0 &&
                 value_batch_stride % 2 == 0 && rope_row_stride % 2 == 0 &&
                 center_batch_stride % 2 == 0,
             "batch strides must be even");
  pg::AppendParams p{};
  p.q = static_cast<const __half*>(query);
  p.k = static_cast<const __half*>(key);
  p.v = static_cast<const __half*>(value);
  p.q_stride_b = query_batch_stride;
  p.k_stride_b = key_batch_stride;
  p.v_stride_b = value_batch_stride;
  p.cos = static_cast<const __half*>(cosine);
  p.sin = static_cast<const __half*>(sine);
  p.device_position = device_position;
  p.position_stride = position_stride;
  p.host_position = position;
  p.rope_row_stride = rope_row_stride;
  p.rope_rows = rope_rows;
  p.rotated_q = static_cast<__half*>(rotated_query);
  p.key_pages = static_cast<__half*>(exact_key_pages);
  p.value_pages = static_cast<__half*>(exact_value_pages);
  p.key_center = static_cast<const __half*>(key_center);
  p.value_center = static_cast<const __half*>(value_center);
  p.center_stride_b = center_batch_stride;
  p.key_codes = static_cast<int8_t*>(key_codes);
  p.value_codes = static_cast<int8_t*>(value_codes);
  p.key_scales = static_cast<__half*>(key_scales);
  p.value_scales = static_cast<__half*>(value_scales);
  p.batch = batch;
  p.hq = query_heads;
  p.hkv = kv_heads;
  p.exact_pages_per_request = exact_ppr;
  p.exact_sink_pages = exact_sink_pages;
  p.code_pages_per_request = code_ppr;
  p.error_flag = device_error_ptr();
  p.inputs_ready = inputs_ready != 0;
  return launch_pdl(pg::pg_rope_append_page_gauge_kernel<false>, dim3(batch * kv_heads * 2),
                    dim3(pg::kAppendThreads), 0, static_cast<cudaStream_t>(stream),
                    "rope_append_page_gauge launch", p);
}

int32_t pg_rope_append_page_gauge(
    const void* query, const void* key, const void* value,
    const void* cosine, const void* sine, const void* key_center,
    const void* value_center, void* rotated_query, void* exact_key_pages,
    void* exact_value_pages, void* key_codes, void* value_codes,
    void* key_scales, void* value_scales, int64_t query_batch_stride,
    int64_t key_batch_stride, int64_t value_batch_stride,
    int64_t center_batch_stride, int32_t batch, int32_t query_heads,
    int32_t kv_heads, int64_t exact_pages, int64_t code_pages,
    int64_t exact_sink_pages, int64_t position,
    const int32_t* device_position, int64_t rope_row_stride,
    int64_t rope_rows, void* stream) {
  return append_page_gauge_impl(
      query, key, value, cosine, sine, key_center, value_center, rotated_query,
      exact_key_pages, exact_value_pages, key_codes, value_codes, key_scales, value_scales,
      query_batch_stride, key_batch_stride, value_batch_stride, center_batch_stride, batch,
      query_heads, kv_heads, exact_pages, code_pages, exact_sink_pages, position,
      device_position, 0, rope_row_stride, rope_rows, stream);
}

int32_t pg_rope_append_page_gauge_served(
    const void* query, const void* key, const void* value, const void* cosine,
    const void* sine, const void* key_center, const void* value_center,
    void* rotated_query, void* exact_key_pages, void* exact_value_pages, void* key_codes,
    void* value_codes, void* key_scales, void* value_scales, void* value_center_out,
    int64_t query_batch_stride, int64_t key_batch_stride, int64_t value_batch_stride,
    int32_t batch, int32_t query_heads, int32_t kv_heads, int64_t num_code_pages,
    int64_t num_exact_pages, int64_t num_centers, const int32_t* positions,
    const int32_t* token_slots, const int32_t* exact_slots, const int32_t* center_rows,
    int64_t rope_row_stride, int64_t rope_rows, void* stream) {
  PG_REQUIRE(batch > 0, "Q/K/V batch sizes must match and be positive");
  PG_REQUIRE(query_heads > 0 && kv_heads > 0 && query_heads % kv_heads == 0,
             "head counts must be positive with Hq a multiple of Hkv");
  PG_REQUIRE(positions != nullptr && token_slots != nullptr && exact_slots != nullptr &&
                 center_rows != nullptr,
             "served append needs device positions, token slots, exact slots and centre rows");
  PG_REQUIRE(value_center_out != nullptr, "served append needs the per-row value centre output");
  PG_REQUIRE(rope_rows > 0, "dynamic RoPE tables must be matching [positions,128] tensors");
  PG_REQUIRE(num_code_pages > 0 && num_exact_pages > 0 && num_centers > 0,
             "pool, sidecar and centre counts must be positive");
  PG_REQUIRE(num_code_pages < (int64_t(1) << 27) && num_exact_pages < (int64_t(1) << 27),
             "pool page count out of range");
  PG_REQUIRE(aligned(query, 4) && aligned(key, 4) && aligned(value, 4) && aligned(cosine, 4) &&
                 aligned(sine, 4) && aligned(key_center, 4) && aligned(value_center, 4) &&
                 aligned(rotated_query, 4) && aligned(value_center_out, 4),
             "tensors must be 4-byte aligned");
  PG_REQUIRE(aligned(exact_key_pages, 16) && aligned(exact_value_pages, 16) &&
                 aligned(key_codes, 8) && aligned(value_codes, 8),
             "exact pages must be 16-byte and INT8 codes 8-byte aligned");
  PG_REQUIRE(query_batch_stride % 2 == 0 && key_batch_stride % 2 == 0 &&
                 value_batch_stride % 2 == 0 && rope_row_stride % 2 == 0,
             "batch strides must be even");
  pg::AppendParams p{};
  p.q = static_cast<const __half*>(query);
  p.k = static_cast<const __half*>(key);
  p.v = static_cast<const __half*>(value);
  p.q_stride_b = query_batch_stride;
  p.k_stride_b = key_batch_stride;
  p.v_stride_b = value_batch_stride;
  p.cos = static_cast<const __half*>(cosine);
  p.sin = static_cast<const __half*>(sine);
  p.device_position = positions;
  p.position_stride = 1;
  p.rope_row_stride = rope_row_stride;
  p.rope_rows = rope_rows;
  p.rotated_q = static_cast<__half*>(rotated_query);
  p.key_pages = static_cast<__half*>(exact_key_pages);
  p.value_pages = static_cast<__half*>(exact_value_pages);
  p.key_center = static_cast<const __half*>(key_center);
  p.value_center = static_cast<const __half*>(value_center);
  p.center_stride_b = static_cast<int64_t>(kv_heads) * pg::kHeadDim;
  p.key_codes = static_cast<int8_t*>(key_codes);
  p.value_codes = static_cast<int8_t*>(value_codes);
  p.key_scales = static_cast<__half*>(key_scales);
  p.value_scales = static_cast<__half*>(value_scales);
  p.batch = batch;
  p.hq = query_heads;
  p.hkv = kv_heads;
  // Positions are bounded by the RoPE table only; the slots carry the pages.
  p.code_pages_per_request = (int64_t(1) << 40);
  p.error_flag = device_error_ptr();
  p.token_slots = token_slots;
  p.exact_slots = exact_slots;
  p.center_rows = center_rows;
  p.center_out = static_cast<__half*>(value_center_out);
  p.num_code_pages = num_code_pages;
  p.num_exact_pages = num_exact_pages;
  p.num_centers = num_centers;
  return launch_pdl(pg::pg_rope_append_page_gauge_kernel<true>, dim3(batch * kv_heads * 2),
                    dim3(pg::kAppendThreads), 0, static_cast<cudaStream_t>(stream),
                    "served rope_append_page_gauge launch", p);
}

int32_t pg_zero_pool_pages(void* key_codes, void* value_codes, void* key_scales,
                           void* value_scales, int64_t num_pages, int32_t kv_heads,
                           const int32_t* page_ids, int32_t count, void* stream) {
  PG_REQUIRE(count >= 0 && num_pages > 0 && kv_heads > 0 && kv_heads <= 256,
             "page counts must be positive and kv_heads in 1..256");
  if (count == 0) return PG_OK;
  PG_REQUIRE(page_ids != nullptr, "page ids are required");
  PG_REQUIRE(aligned(key_codes, 16) && aligned(value_codes, 16) && aligned(key_scales, 2) &&
                 aligned(value_scales, 2),
             "code planes must be 16-byte aligned");
  pg::pg_zero_pool_pages_kernel<<<static_cast<unsigned>(count), 256, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
      static_cast<int8_t*>(key_codes), static_cast<int8_t*>(value_codes),
      static_cast<__half*>(key_scales), static_cast<__half*>(value_scales), num_pages, kv_heads,
      page_ids, device_error_ptr());
  return cuda_check(cudaGetLastError(), "zero pool pages launch");
}

int32_t pg_rope_append_page_gauge_batched(
    const void* query, const void* key, const void* value,
    const void* cosine, const void* sine, const void* key_center,
    const void* value_center, void* rotated_query, void* exact_key_pages,
    void* exact_value_pages, void* key_codes, void* value_codes,
    void* key_scales, void* value_scales, int64_t query_batch_stride,
    int64_t key_batch_stride, int64_t value_batch_stride,
    int64_t center_batch_stride, int32_t batch, int32_t query_heads,
    int32_t kv_heads, int64_t exact_pages, int64_t code_pages,
    int64_t exact_sink_pages, const int32_t* positions,
    int64_t rope_row_stride, int64_t rope_rows, int32_t inputs_ready, void* stream) {
  PG_REQUIRE(positions != nullptr, "per-request positions must be a device int32 [B] tensor");
  return append_page_gauge_impl(
      query, key, value, cosine, sine, key_center, value_center, rotated_query,
      exact_key_pages, exact_value_pages, key_codes, value_codes, key_scales, value_scales,
      query_batch_stride, key_batch_stride, value_batch_stride, center_batch_stride, batch,
      query_heads, kv_heads, exact_pages, code_pages, exact_sink_pages, 0, positions, 1,
      rope_row_stride, rope_rows, stream, inputs_ready);
}

// -------------------------------------------------------------- tail merge
int32_t pg_exact_tail_merge_center(
    const void* query, const void* exact_key_pages,
    const void* exact_value_pages, int64_t exact_pages_total,
    const int32_t* exact_page_indices, int64_t num_indices,
    const int32_t* exact_last_page_len, void* old_output, float* old_lse,
    const void* value_center, int64_t center_batch_stride, int32_t batch,
    int32_t query_heads, int32_t kv_heads, double sm_scale, void* stream) {
  PG_REQUIRE(batch > 0, "batch size must be positive");
  PG_REQUIRE(query_heads > 0 && kv_heads > 0 && query_heads % kv_heads == 0,
             "query heads must be a positive multiple of KV heads");
  PG_REQUIRE(query_heads / kv_heads <= 8,
             "the fused exact-tail kernel supports GQA group sizes up to 8");
  PG_REQUIRE(num_indices % batch == 0, "exact page indices must divide evenly across requests");
  const int64_t n = num_indices / batch;
  PG_REQUIRE(n > 0 && n <= 16, "the fused exact tail supports 1..16 pages per request");
  PG_REQUIRE(exact_pages_total >= batch * n, "exact page index count exceeds the ring allocation");
  PG_REQUIRE(sm_scale > 0.0 && std::isfinite(sm_scale), "sm_scale must be positive and finite");
  PG_REQUIRE(aligned(exact_key_pages, 16) && aligned(exact_value_pages, 16),
             "exact caches must be 16-byte aligned");
  pg::DecodeParams p{};
  p.q = static_cast<const __half*>(query);
  p.q_stride_b = static_cast<int64_t>(query_heads) * pg::kHeadDim;
  p.q_stride_h = pg::kHeadDim;
  p.seg[1].indices = exact_page_indices;
  p.seg[1].last_len = exact_last_page_len;
  p.seg[1].num_pages = static_cast<int32_t>(exact_pages_total);
  p.items = nullptr;
  p.num_items = batch * kv_heads;
  p.hkv = kv_heads;
  p.group = query_heads / kv_heads;
  p.sm_scale_log2 = static_cast<float>(sm_scale) * 1.4426950408889634f;
  p.final_mode = 1;
  p.out = static_cast<__half*>(old_output);
  p.out_stride_b = static_cast<int64_t>(query_heads) * pg::kHeadDim;
  p.out_stride_h = pg::kHeadDim;
  p.lse_out = old_lse;
  p.extra_o = static_cast<const __half*>(old_output);
  p.extra_stride_b = p.out_stride_b;
  p.extra_stride_h = p.out_stride_h;
  p.extra_lse = old_lse;
  p.value_center = static_cast<const __half*>(value_center);
  p.vc_stride_b = center_batch_stride;
  p.implicit_pages = static_cast<int32_t>(n);
  p.sem = nullptr;
  p.item_off = nullptr;
  p.error_flag = device_error_ptr();
  CUtensorMap k16, v16, none;
  std::memset(&none, 0, sizeof(none));
  int32_t rc = make_page_map(&k16, exact_key_pages, exact_pages_total, kv_heads, true);
  if (rc != PG_OK) return rc;
  rc = make_page_map(&v16, exact_value_pages, exact_pages_total, kv_heads, true);
  if (rc != PG_OK) return rc;
  const int warps = n >= 8 ? 8 : static_cast<int>(n);
  return launch_decode(p, none, none, k16, v16, batch * kv_heads, warps,
                       static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ decode
int32_t pg_decode_plan(int32_t batch, int32_t kv_heads, const int32_t* indptr0,
                       const int32_t* indptr1, int32_t split_pages0,
                       int32_t split_pages1, int32_t num_sms,
                       int32_t warps_per_cta, pg_decode_item* items,
                       int64_t items_capacity, int32_t* item_off,
                       pg_plan_info* info) {
  PG_REQUIRE(batch > 0 && kv_heads > 0, "batch and kv heads must be positive");
  PG_REQUIRE(indptr0 != nullptr || indptr1 != nullptr, "at least one segment is required");
  PG_REQUIRE(split_pages0 >= 0 && split_pages1 >= 0, "fixed split size must be non-negative");
  PG_REQUIRE(kv_heads < 65536, "too many kv heads");
  const int W = warps_per_cta <= 0 ? 4 : std::min(warps_per_cta, pg::kMaxWarps);
  const int32_t* ind[2] = {indptr0, indptr1};
  int64_t pages[2] = {0, 0};
  for (int s = 0; s < 2; ++s) {
    if (ind[s] == nullptr) continue;
    PG_REQUIRE(ind[s][0] >= 0, "indptr must start at a non-negative offset");
    for (int r = 0; r < batch; ++r) {
      const int64_t n = static_cast<int64_t>(ind[s][r + 1]) - ind[s][r];
      PG_REQUIRE(n >= 0, "indptr must be non-decreasing");
      pages[s] += n;
    }
  }
  int split[2] = {split_pages0, split_pages1};
  // A given INT8 split with an automatic FP16 split: FP16 items of the same
  // bytes (an FP16 page moves twice an INT8 page's), so the tail does not
  // break into many short items that push the plan past one wave.
  if (split[0] > 0 && split[1] == 0) split[1] = std::max(1, split[0] / 2);
  if (split[0] == 0 || split[1] == 0) {
    // Automatic: minimise the estimated makespan
    //   ceil(items / resident_slots) * (pages per item + startup overhead)
    // where an FP16 page counts twice an INT8 page and an FP16 item gets
    // half the pages.  One full wave (items <= slots) is what this usually
    // picks; a partial second wave doubles the step time.
    const int ctas_per_sm = pg_ctas_per_sm(W);
    const int64_t slots = static_cast<int64_t>(std::max(num_sms, 1)) * ctas_per_sm;
    int64_t max_n = 1;
    for (int s = 0; s < 2; ++s) {
      if (ind[s] == nullptr) continue;
      for (int r = 0; r < batch; ++r)
        max_n = std::max<int64_t>(max_n, static_cast<int64_t>(ind[s][r + 1]) - ind[s][r]);
    }
    constexpr double kOverheadPages = 8.0;  // ~2 us of CTA start-up at 15 GB/s
    double best_cost = 1e300;
    int best = 1;
    for (int64_t c = 1; c <= std::min<int64_t>(max_n, 32 * W); c = c < 64 ? c + 1 : c + c / 32) {
      const int64_t c0 = split[0] ? split[0] : c;
      const int64_t c1 = split[1] ? split[1] : std::max<int64_t>(1, c / 2);
      int64_t items = 0;
      double longest = 0.0;
      for (int r = 0; r < batch; ++r) {
        for (int s = 0; s < 2; ++s) {
          if (ind[s] == nullptr) continue;
          const int64_t n = static_cast<int64_t>(ind[s][r + 1]) - ind[s][r];
          const int64_t cs = s == 0 ? c0 : c1;
          items += (n + cs - 1) / cs;
          longest = std::max(longest, static_cast<double>(std::min(n, cs)) * (s == 0 ? 1.0 : 2.0));
        }
      }
      items *= kv_heads;
      const double waves = static_cast<double>((items + slots - 1) / slots);
      const double cost = waves * (longest + kOverheadPages);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = static_cast<int>(c);
      }
    }
    if (split[0] == 0) split[0] = best;
    if (split[1] == 0) split[1] = std::max(1, best / 2);
  }
  // At most 32 pages per warp: the kernel keeps a warp's page ids and scales
  // in one register window.
  split[0] = std::min(split[0], 32 * W);
  split[1] = std::min(split[1], 32 * W);
  int64_t count = 0;
  int32_t max_per_head = 0;
  bool single = true;
  for (int r = 0; r < batch; ++r) {
    for (int h = 0; h < kv_heads; ++h) {
      if (item_off) item_off[r * kv_heads + h] = static_cast<int32_t>(count);
      int32_t here = 0;
      for (int s = 0; s < 2; ++s) {
        if (ind[s] == nullptr) continue;
        const int32_t b = ind[s][r], e = ind[s][r + 1];
        for (int32_t c = b; c < e; c += split[s]) {
          const int32_t n = std::min(split[s], e - c);
          if (count < items_capacity && items != nullptr) {
            pg_decode_item& it = items[count];
            it.request = r;
            it.head_seg = h | (s << 16);
            it.idx_begin = c;
            it.count = n | ((c + n == e) ? static_cast<int32_t>(0x80000000u) : 0);
          }
          ++count;
          ++here;
        }
      }
      max_per_head = std::max(max_per_head, here);
      if (here != 1) single = false;
    }
  }
  if (item_off) item_off[batch * kv_heads] = static_cast<int32_t>(count);
  if (info) {
    info->num_items = count;
    info->max_items_per_head = max_per_head;
    info->single_item_per_head = single ? 1 : 0;
    info->split_pages[0] = split[0];
    info->split_pages[1] = split[1];
    info->warps_per_cta = W;
  }
  if (count > items_capacity)
    return fail(PG_ERR_CAPACITY, "work list needs %lld items, capacity %lld",
                static_cast<long long>(count), static_cast<long long>(items_capacity));
  PG_REQUIRE(count < (int64_t(1) << 31), "too many work items");
  return PG_OK;
}

int32_t pg_decode_run(const pg_decode_args* a, void* stream) {
  PG_REQUIRE(a != nullptr, "null arguments");
  PG_REQUIRE(a->batch > 0 && a->kv_heads > 0, "batch and kv heads must be positive");
  PG_REQUIRE(a->group >= 1 && a->group <= 8, "GQA group size must be in 1..8");
  PG_REQUIRE(a->sm_scale > 0.f && std::isfinite(a->sm_scale), "sm_scale must be positive and finite");
  PG_REQUIRE(a->q != nullptr && aligned(a->q, 4) && a->q_stride_b % 2 == 0 && a->q_stride_h % 2 == 0,
             "query must be 4-byte aligned with even strides");
  PG_REQUIRE(a->out != nullptr, "output is required");
  PG_REQUIRE(a->num_items >= 0, "negative item count");
  const int W = a->warps_per_cta <= 0 ? 4 : std::min(a->warps_per_cta, pg::kMaxWarps);
  PG_REQUIRE(a->representation == 0 || a->representation == 1,
             "representation must be 0 (page gauge) or 1 (affine_group16)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  pg::DecodeParams p{};
  p.k_bias = static_cast<const __half*>(a->k_bias);
  p.v_bias = static_cast<const __half*>(a->v_bias);
  p.q = static_cast<const __half*>(a->q);
  p.q_stride_b = a->q_stride_b;
  p.q_stride_h = a->q_stride_h;
  CUtensorMap maps[4];
  std::memset(maps, 0, sizeof(maps));
  for (int s = 0; s < 2; ++s) {
    const pg_segment& sg = a->seg[s];
    if (sg.k_cache == nullptr) continue;
    PG_REQUIRE(sg.v_cache != nullptr && sg.indices != nullptr && sg.last_page_len != nullptr,
               "segment %d is incomplete", s);
    PG_REQUIRE(sg.num_pages > 0 && sg.num_pages < (int64_t(1) << 27),
               "segment %d page count out of range", s);
    if (s == 0)
      PG_REQUIRE(sg.k_scale != nullptr && sg.v_scale != nullptr,
                 "INT8 segment needs k/v page scales");
    if (s == 0 && a->representation == 1)
      PG_REQUIRE(aligned(sg.k_scale, 16) && aligned(sg.v_scale, 16) && a->k_bias != nullptr &&
                     a->v_bias != nullptr && aligned(a->k_bias, 16) && aligned(a->v_bias, 16),
                 "affine_group16 needs 16-byte aligned [pages,Hkv,8] group scales and biases");
    int32_t rc = make_page_map(&maps[2 * s], sg.k_cache, sg.num_pages, a->kv_heads, s == 1);
    if (rc != PG_OK) return rc;
    rc = make_page_map(&maps[2 * s + 1], sg.v_cache, sg.num_pages, a->kv_heads, s == 1);
    if (rc != PG_OK) return rc;
    p.seg[s].indices = sg.indices;
    p.seg[s].last_len = sg.last_page_len;
    p.seg[s].k_scale = static_cast<const __half*>(sg.k_scale);
    p.seg[s].v_scale = static_cast<const __half*>(sg.v_scale);
    p.seg[s].num_pages = static_cast<int32_t>(sg.num_pages);
  }
  p.items = reinterpret_cast<const pg::DecodeItem*>(a->items);
  p.num_items = a->num_items;
  p.hkv = a->kv_heads;
  p.group = a->group;
  p.sm_scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.part_o = a->part_o;
  p.part_lse = a->part_lse;
  p.final_mode = a->final_mode;
  p.out = static_cast<__half*>(a->out);
  p.out_stride_b = a->out_stride_b;
  p.out_stride_h = a->out_stride_h;
  p.lse_out = a->lse_out;
  p.extra_o = static_cast<const __half*>(a->extra_o);
  p.extra_stride_b = a->extra_stride_b;
  p.extra_stride_h = a->extra_stride_h;
  p.extra_lse = a->extra_lse;
  p.value_center = static_cast<const __half*>(a->value_center);
  p.vc_stride_b = a->vc_stride_b;
  p.implicit_pages = 0;
  p.int8_after_wait = a->int8_after_wait != 0;
  p.error_flag = device_error_ptr();
  const bool fused = a->merge_sem != nullptr && !a->final_mode;
  p.sem = fused ? a->merge_sem : nullptr;
  p.item_off = a->item_off;
  if (fused) PG_REQUIRE(a->item_off != nullptr, "the fused merge needs item offsets");
  PG_REQUIRE(a->cluster >= 0 && a->cluster <= 8, "cluster size must be 0..8");
  const int cluster = (fused && a->cluster > 1) ? a->cluster : 1;
  p.cluster = cluster;
  if (cluster > 1) {
    PG_REQUIRE(W >= 2, "the cluster merge needs at least 2 warps per CTA");
  }
  if (a->extra_o != nullptr) PG_REQUIRE(a->extra_lse != nullptr, "extra state needs its lse");

  const int mask = (a->stage_mask & 3) == 0 ? 3 : (a->stage_mask & 3);
  if (a->num_items > 0 && (mask & 1)) {
    PG_REQUIRE(a->items != nullptr, "work items are required");
    if (!a->final_mode)
      PG_REQUIRE(a->part_o != nullptr && a->part_lse != nullptr,
                 "split decode needs a partial-state workspace");
    const int ctas = (a->num_items + cluster - 1) / cluster * cluster;
    int32_t rc = launch_decode(p, maps[0], maps[1], maps[2], maps[3], ctas, W, st, cluster,
                               a->representation == 1 ? pg::kRepAffine16 : pg::kRepGauge);
    if (rc != PG_OK) return rc;
  }
  if (a->final_mode && a->num_items > 0) return PG_OK;
  if (fused && a->num_items > 0 && (mask & 1)) return PG_OK;
  if (!(mask & 2)) return PG_OK;

  PG_REQUIRE(a->item_off != nullptr, "item offsets are required for the merge");
  pg::MergeParams m{};
  m.part_o = a->part_o;
  m.part_lse = a->part_lse;
  m.item_off = a->item_off;
  m.batch = a->batch;
  m.hkv = a->kv_heads;
  m.group = a->group;
  m.out = p.out;
  m.out_stride_b = a->out_stride_b;
  m.out_stride_h = a->out_stride_h;
  m.lse_out = a->lse_out;
  m.extra_o = p.extra_o;
  m.extra_stride_b = a->extra_stride_b;
  m.extra_stride_h = a->extra_stride_h;
  m.extra_lse = a->extra_lse;
  m.value_center = p.value_center;
  m.vc_stride_b = a->vc_stride_b;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a->batch * a->kv_heads * a->group);
  cfg.blockDim = dim3(pg::kMergeWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, pg::pg_merge_partials_kernel, m),
                    "merge kernel launch");
}

int32_t pg_decode_max_clusters(int32_t warps, int32_t cluster, int32_t* out) {
  PG_REQUIRE(out != nullptr && warps >= 1 && warps <= pg::kMaxWarps && cluster >= 1 && cluster <= 8,
             "bad arguments");
  int32_t rc = ensure_decode_smem();
  if (rc != PG_OK) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(cluster * 64);
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = pg::decode_smem_bytes(warps);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  rc = cuda_check(cudaOccupancyMaxActiveClusters(&n, pg::pg_decode_split_kernel<pg::kRepGauge, false>, &cfg),
                  "cudaOccupancyMaxActiveClusters");
  if (rc != PG_OK) return rc;
  *out = n;
  return PG_OK;
}

int32_t pg_merge_state_in_place(void* v_a, float* s_a, const void* v_b,
                                const float* s_b, int64_t rows,
                                int64_t va_row_stride, int64_t vb_row_stride,
                                void* stream) {
  PG_REQUIRE(rows >= 0, "rows must be non-negative");
  if (rows == 0) return PG_OK;
  PG_REQUIRE(rows < (int64_t(1) << 31), "too many rows");
  pg::pg_merge_state_kernel<<<static_cast<unsigned>(rows), 128, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(v_a), s_a, static_cast<const __half*>(v_b), s_b, rows,
      va_row_stride, vb_row_stride);
  return cuda_check(cudaGetLastError(), "merge_state launch");
}

int32_t pg_quantize_pages(const void* key, const void* value,
                          const void* key_center, const void* value_center,
                          int64_t pages_per_center, void* key_codes,
                          void* value_codes, void* key_scales,
                          void* value_scales, int64_t num_pages,
                          int32_t kv_heads, int32_t rounding, void* stream) {
  PG_REQUIRE(num_pages >= 0 && kv_heads > 0, "page and head counts must be positive");
  PG_REQUIRE(rounding == 0 || rounding == 1, "rounding must be 0 (half away) or 1 (half even)");
  PG_REQUIRE(pages_per_center >= 0, "pages_per_center must be non-negative");
  if (num_pages == 0) return PG_OK;
  PG_REQUIRE(num_pages * kv_heads < (int64_t(1) << 31), "too many pages");
  const bool key_only = value == nullptr;
  PG_REQUIRE(!key_only || (value_center == nullptr && value_codes == nullptr &&
                           value_scales == nullptr),
             "value, value_center, value_codes and value_scales are all given or all NULL");
  PG_REQUIRE(key != nullptr && key_center != nullptr && key_codes != nullptr &&
                 key_scales != nullptr,
             "key, key_center, key_codes and key_scales are required");
  PG_REQUIRE(aligned(key, 4) && aligned(value, 4) && aligned(key_center, 4) &&
                 aligned(value_center, 4) && aligned(key_codes, 2) && aligned(value_codes, 2),
             "tensors must be aligned");
  pg::QuantizeParams p{};
  p.key = static_cast<const __half*>(key);
  p.value = static_cast<const __half*>(value);
  p.key_center = static_cast<const __half*>(key_center);
  p.value_center = static_cast<const __half*>(value_center);
  p.pages_per_center = pages_per_center;
  p.key_codes = static_cast<int8_t*>(key_codes);
  p.value_codes = static_cast<int8_t*>(value_codes);
  p.key_scales = static_cast<__half*>(key_scales);
  p.value_scales = static_cast<__half*>(value_scales);
  p.num_pages = num_pages;
  p.hkv = kv_heads;
  p.half_even = rounding;
  pg::pg_quantize_pages_kernel<<<static_cast<unsigned>(num_pages * kv_heads), 64, 0,
                                 static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_check(cudaGetLastError(), "quantize launch");
}

int32_t pg_quantize_affine_group16(const void* values, int64_t num_pages, int32_t kv_heads,
                                   void* codes, void* bias, void* scale, void* reconstructed,
                                   void* stream) {
  PG_REQUIRE(num_pages >= 0 && kv_heads > 0, "page and head counts must be positive");
  if (num_pages == 0) return PG_OK;
  PG_REQUIRE(num_pages * kv_heads < (int64_t(1) << 31), "too many pages");
  PG_REQUIRE(values != nullptr && codes != nullptr && bias != nullptr && scale != nullptr,
             "values, codes, bias and scale are required");
  PG_REQUIRE(aligned(values, 8) && aligned(codes, 4) && aligned(bias, 2) && aligned(scale, 2) &&
                 aligned(reconstructed, 8),
             "tensors must be aligned");
  pg::AffineQuantParams p{};
  p.values = static_cast<const __half*>(values);
  p.codes = static_cast<int8_t*>(codes);
  p.bias = static_cast<__half*>(bias);
  p.scale = static_cast<__half*>(scale);
  p.recon = static_cast<__half*>(reconstructed);
  p.num_pages = num_pages;
  p.hkv = kv_heads;
  const int64_t warps = num_pages * kv_heads;
  const unsigned blocks =
      static_cast<unsigned>((warps + pg::kAffineQuantWarps - 1) / pg::kAffineQuantWarps);
  pg::pg_quantize_affine_kernel<<<blocks, pg::kAffineQuantWarps * 32, 0,
                                  static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_check(cudaGetLastError(), "affine quantize launch");
}

// ------------------------------------------------ decoder layer element-wise
int32_t pg_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out,
                       int32_t rows, int32_t hidden, int64_t residual_stride,
                       int64_t delta_stride, int64_t out_stride, float eps, void* stream) {
  PG_REQUIRE(rows > 0, "rows must be positive");
  PG_REQUIRE(hidden > 0 && hidden % 8 == 0 && hidden <= 4 * 8 * pg::kNormThreads,
             "hidden size must be a positive multiple of 8 up to 16384");
  PG_REQUIRE(residual_stride % 8 == 0 && out_stride % 8 == 0 && (delta == nullptr || delta_stride % 8 == 0),
             "row strides must be multiples of 8 elements");
  PG_REQUIRE(aligned(residual, 16) && aligned(weight, 16) && aligned(out, 16) &&
                 (delta == nullptr || aligned(delta, 16)),
             "tensors must be 16-byte aligned");
  PG_REQUIRE(eps > 0.f && std::isfinite(eps), "eps must be positive");
  pg::NormParams p{};
  p.residual = static_cast<__half*>(residual);
  p.delta = static_cast<const __half*>(delta);
  p.weight = static_cast<const __half*>(weight);
  p.out = static_cast<__half*>(out);
  p.residual_stride = residual_stride;
  p.delta_stride = delta_stride;
  p.out_stride = out_stride;
  p.hidden = hidden;
  p.eps = eps;
  return launch_pdl(pg::pg_add_rmsnorm_kernel, dim3(rows), dim3(pg::kNormThreads), 0,
                    static_cast<cudaStream_t>(stream), "add_rmsnorm launch", p);
}

int32_t pg_silu_mul(const void* gate_up, void* out, int32_t rows, int32_t features,
                    int64_t in_stride, int64_t out_stride, void* stream) {
  PG_REQUIRE(rows > 0 && features > 0 && features % 8 == 0,
             "rows must be positive and features a positive multiple of 8");
  PG_REQUIRE(in_stride % 8 == 0 && out_stride % 8 == 0 && in_stride >= 2 * static_cast<int64_t>(features),
             "row strides must be multiples of 8 elements and hold gate and up");
  PG_REQUIRE(aligned(gate_up, 16) && aligned(out, 16), "tensors must be 16-byte aligned");
  pg::SiluMulParams p{};
  p.gate_up = static_cast<const __half*>(gate_up);
  p.out = static_cast<__half*>(out);
  p.in_stride = in_stride;
  p.out_stride = out_stride;
  p.rows = rows;
  p.features = features;
  const int64_t chunks = static_cast<int64_t>(rows) * (features / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148 * 8));
  return launch_pdl(pg::pg_silu_mul_kernel, dim3(blocks), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), "silu_mul launch", p);
}

int32_t pg_step_positions(int32_t* positions, int32_t* last_page_len, int32_t batch,
                          int32_t advance, void* stream) {
  PG_REQUIRE(positions != nullptr && batch > 0, "positions must be a device int32 [B] tensor");
  return launch_pdl(pg::pg_step_positions_kernel, dim3((batch + 127) / 128), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), "step_positions launch", positions,
                    last_page_len, batch, advance);
}

int32_t pg_argmax_rows(const void* logits, int64_t ld, int32_t rows, int32_t cols,
                       int64_t index_offset, float* out_val, int64_t* out_idx, void* stream) {
  PG_REQUIRE(rows > 0 && cols > 0 && cols % 8 == 0, "rows must be positive and cols a positive multiple of 8");
  PG_REQUIRE(ld % 8 == 0 && ld >= cols && aligned(logits, 16), "logit rows must be 16-byte aligned");
  PG_REQUIRE(out_idx != nullptr, "out_idx is required");
  return launch_pdl(pg::pg_argmax_rows_kernel, dim3(rows), dim3(pg::kArgmaxThreads), 0,
                    static_cast<cudaStream_t>(stream), "argmax launch",
                    static_cast<const __half*>(logits), ld, cols, index_offset, out_val, out_idx);
}

// ------------------------------------------------------- skinny GEMM
namespace {

int32_t make_2d_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows,
                    int64_t row_stride_elems, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(PG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(pg::kGemmBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return PG_OK;
}

int gemm_nt(int batch) { return batch <= 8 ? 1 : (batch <= 16 ? 2 : 4); }

// Static shared memory of the kernel (epilogue tile) plus 1 KB per CTA.
int gemm_ctas_per_sm(int nt) {
  const int stat = pg::kGemmTileRows * (8 * nt + 1) * 4 + 16;
  return std::max(1, (228 * 1024) / (pg::gemm_smem_bytes(nt) + stat + 1024));
}

struct GemmShape {
  int32_t tiles, kblocks, grid, max_seg, total;
};

int32_t gemm_shape(int32_t n, int32_t k, int32_t batch, int32_t mode, int32_t grid,
                   int32_t num_sms, GemmShape* out) {
  PG_REQUIRE(batch >= 1 && batch <= 32, "batch must be 1..32");
  PG_REQUIRE(k > 0 && k % pg::kGemmBK == 0, "k must be a positive multiple of 64");
  PG_REQUIRE(mode >= 0 && mode <= 2, "mode must be 0 (store), 1 (residual) or 2 (silu_mul)");
  if (mode == pg::kGemmSiluMul)
    PG_REQUIRE(n > 0 && n % 64 == 0, "silu_mul needs n (gate + up rows) a positive multiple of 64");
  else
    PG_REQUIRE(n > 0 && n % pg::kGemmTileRows == 0, "n must be a positive multiple of 64");
  GemmShape g{};
  g.tiles = mode == pg::kGemmSiluMul ? (n / 2) / 32 : n / pg::kGemmTileRows;
  g.kblocks = k / pg::kGemmBK;
  const int64_t total = static_cast<int64_t>(g.tiles) * g.kblocks;
  const int64_t slots = static_cast<int64_t>(std::max(num_sms, 1)) * gemm_ctas_per_sm(gemm_nt(batch));
  // Default grid: every resident CTA slot, except for narrow shapes (at
  // most 1024 weight blocks of 64 x 64, e.g. a tensor-parallel rank's
  // qkv / o projection at TP8), which one CTA per SM streams faster
  // (TP8 B=1: qkv 7.55 -> 6.75 us, o 7.16 -> 5.96 us).
  const int64_t fallback = total <= 1024 ? std::max(num_sms, 1) : slots;
  int64_t grid_n = std::min<int64_t>(total, grid > 0 ? grid : fallback);
  // At most 16 CTAs may share a tile (the finishing CTA's slot table).
  while (grid_n > 1 && (g.kblocks + total / grid_n - 1) / (total / grid_n) + 1 > pg::kGemmMaxContrib)
    --grid_n;
  PG_REQUIRE(total * grid_n < (int64_t(1) << 31), "GEMM too large for the stream-K indexing");
  g.total = static_cast<int32_t>(total);
  g.grid = static_cast<int32_t>(grid_n);
  const int64_t lmax = (total + grid_n - 1) / grid_n;
  g.max_seg = static_cast<int32_t>((g.kblocks - 1 + lmax + g.kblocks - 1) / g.kblocks);
  *out = g;
  return PG_OK;
}

int32_t ensure_gemm_smem() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(PG_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    int32_t rc = PG_OK;
    auto set = [&](auto kernel, int nt) {
      if (rc == PG_OK)
        rc = cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             pg::gemm_smem_bytes(nt)),
                        "cudaFuncSetAttribute(gemm)");
    };
    set(pg::pg_skinny_gemm_kernel<1, false>, 1);
    set(pg::pg_skinny_gemm_kernel<2, false>, 2);
    set(pg::pg_skinny_gemm_kernel<4, false>, 4);
    set(pg::pg_skinny_gemm_kernel<1, true>, 1);
    set(pg::pg_skinny_gemm_kernel<2, true>, 2);
    set(pg::pg_skinny_gemm_kernel<4, true>, 4);
    if (rc != PG_OK) return rc;
    done[dev] = true;
  }
  return PG_OK;
}

int current_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

int32_t pg_skinny_gemm_workspace(int32_t n, int32_t k, int32_t batch, int32_t mode, int32_t grid,
                                 int32_t num_sms, int64_t* partial_floats, int32_t* counters) {
  GemmShape g;
  int32_t rc = gemm_shape(n, k, batch, mode, grid, num_sms > 0 ? num_sms : current_sms(), &g);
  if (rc != PG_OK) return rc;
  if (partial_floats != nullptr)
    *partial_floats = static_cast<int64_t>(g.grid) * g.max_seg * pg::kGemmTileRows * 8 * gemm_nt(batch);
  if (counters != nullptr) *counters = g.tiles;
  return PG_OK;
}

int32_t pg_pack_weight(const void* w, int64_t ld, int32_t n, int32_t k, int32_t mode, void* out,
                       void* stream) {
  PG_REQUIRE(k > 0 && k % pg::kGemmBK == 0 && n > 0 && n % 64 == 0,
             "n and k must be positive multiples of 64");
  PG_REQUIRE(mode >= 0 && mode <= 2, "mode must be 0, 1 or 2");
  PG_REQUIRE(ld >= k && ld % 8 == 0 && aligned(w, 16) && aligned(out, 16),
             "w rows must be 16-byte aligned and cover k");
  const int64_t chunks = static_cast<int64_t>(n) * (k / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148 * 16));
  pg::pg_pack_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), ld, n, k, mode, static_cast<__half*>(out));
  return cuda_check(cudaGetLastError(), "pack_weight launch");
}

int32_t pg_skinny_gemm(const pg_gemm_args* a, void* stream) {
  PG_REQUIRE(a != nullptr, "null arguments");
  GemmShape g;
  int32_t rc = gemm_shape(a->n, a->k, a->batch, a->mode, a->grid, current_sms(), &g);
  if (rc != PG_OK) return rc;
  const int nt = gemm_nt(a->batch);
  PG_REQUIRE(a->w != nullptr && a->x != nullptr, "w and x are required");
  PG_REQUIRE(aligned(a->w, 16) && aligned(a->x, 16), "w and x must be 16-byte aligned");
  PG_REQUIRE(a->ldx >= a->k && a->ldx % 8 == 0,
             "the x row stride must cover k and be a multiple of 8 elements");
  if (a->tp_world > 1)
    PG_REQUIRE(a->mode == pg::kGemmStore,
               "a tensor-parallel GEMM publishes its tiles (store mode); pg_tp_reduce applies "
               "the epilogue");
  else if (a->mode == pg::kGemmResidual)
    PG_REQUIRE(a->residual != nullptr && a->ldr >= a->n, "residual mode needs residual [batch, n]");
  else
    PG_REQUIRE(a->y != nullptr && a->ldy >= (a->mode == pg::kGemmSiluMul ? a->n / 2 : a->n),
               "y [batch, n] (silu_mul: [batch, n/2]) is required");
  const int64_t need = static_cast<int64_t>(g.grid) * g.max_seg * pg::kGemmTileRows * 8 * nt;
  PG_REQUIRE(a->partials != nullptr && a->partial_floats >= need && a->counters != nullptr &&
                 a->num_counters >= g.tiles,
             "split-K workspace too small (query pg_skinny_gemm_workspace)");
  rc = ensure_gemm_smem();
  if (rc != PG_OK) return rc;
  CUtensorMap tx;
  rc = make_2d_map(&tx, a->x, a->k, a->batch, a->ldx, 8 * nt);
  if (rc != PG_OK) return rc;
  pg::GemmParams p{};
  p.n = a->n;
  p.k = a->k;
  p.batch = a->batch;
  p.mode = a->mode;
  p.tiles = g.tiles;
  p.kblocks = g.kblocks;
  p.total = g.total;
  p.grid = g.grid;
  p.max_seg = g.max_seg;
  p.half_rows = a->n / 2;
  p.y = static_cast<__half*>(a->y);
  p.ldy = a->ldy;
  p.residual = static_cast<__half*>(a->residual);
  p.ldr = a->ldr;
  p.partials = a->partials;
  p.counters = a->counters;
  p.error_flag = device_error_ptr();
  p.tp_world = 1;
  if (a->tp_world > 1) {
    PG_REQUIRE(a->tp_world <= pg::kGemmMaxTp && a->tp_rank >= 0 && a->tp_rank < a->tp_world,
               "tensor-parallel world must be 2..8 with 0 <= rank < world");
    PG_REQUIRE(a->tp_tiles_cap >= g.tiles, "exchange buffers hold fewer tiles than the output");
    for (int r = 0; r < a->tp_world; ++r)
      PG_REQUIRE(a->tp_peers[r] != nullptr && aligned(a->tp_peers[r], 256),
                 "every rank's exchange buffer is required");
    p.tp_world = a->tp_world;
    p.tp_rank = a->tp_rank;
    p.tp_tiles_cap = a->tp_tiles_cap;
    for (int r = 0; r < a->tp_world; ++r) p.tp_peers[r] = static_cast<uint8_t*>(a->tp_peers[r]);
  }
  if (a->norm_weight != nullptr) {
    PG_REQUIRE(aligned(a->norm_weight, 16), "the norm weight must be 16-byte aligned");
    PG_REQUIRE(a->norm_eps > 0.f && std::isfinite(a->norm_eps), "norm eps must be positive");
    p.norm_w = static_cast<const __half*>(a->norm_weight);
    p.x = static_cast<const __half*>(a->x);
    p.ldx = a->ldx;
    p.norm_eps = a->norm_eps;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(g.grid);
  cfg.blockDim = dim3(pg::kGemmWarps * 32);
  cfg.dynamicSmemBytes = pg::gemm_smem_bytes(nt);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a->pdl ? 1 : 0;
  const __half* wp = static_cast<const __half*>(a->w);
  const bool norm = p.norm_w != nullptr;
  cudaError_t e;
  if (nt == 1)
    e = norm ? cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<1, true>, wp, tx, p)
             : cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<1, false>, wp, tx, p);
  else if (nt == 2)
    e = norm ? cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<2, true>, wp, tx, p)
             : cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<2, false>, wp, tx, p);
  else
    e = norm ? cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<4, true>, wp, tx, p)
             : cudaLaunchKernelEx(&cfg, pg::pg_skinny_gemm_kernel<4, false>, wp, tx, p);
  return cuda_check(e, "skinny gemm launch");
}

int32_t pg_tp_publish(void* const* peers, int32_t world, int32_t rank, int32_t tiles_cap,
                      int32_t tiles, int32_t batch, const void* src, int64_t src_stride,
                      void* stream) {
  PG_REQUIRE(peers != nullptr, "the ranks' exchange buffers are required");
  PG_REQUIRE(world >= 2 && world <= pg::kGemmMaxTp && rank >= 0 && rank < world,
             "world must be 2..8 with 0 <= rank < world");
  PG_REQUIRE(tiles >= 1 && tiles <= tiles_cap, "tiles must be 1..tiles_cap");
  PG_REQUIRE(batch >= 1 && batch <= pg::kGemmMaxXR, "batch must be 1..32");
  PG_REQUIRE(src != nullptr && aligned(src, 4) && src_stride >= int64_t(tiles) * 64 &&
                 src_stride % 2 == 0,
             "src must be fp16 [batch, tiles * 64] with 4-byte aligned rows");
  pg::TpPublishParams p{};
  for (int r = 0; r < world; ++r) {
    PG_REQUIRE(peers[r] != nullptr && aligned(peers[r], 256),
               "every rank's exchange buffer is required");
    p.peers[r] = static_cast<uint8_t*>(peers[r]);
  }
  p.world = world;
  p.rank = rank;
  p.cap = tiles_cap;
  p.batch = batch;
  p.src = static_cast<const __half*>(src);
  p.src_stride = src_stride;
  return launch_pdl(pg::pg_tp_publish_kernel, dim3(tiles), dim3(pg::kTpPublishThreads), 0,
                    static_cast<cudaStream_t>(stream), "tp publish launch", p);
}

int32_t pg_tp_reduce(const void* exchange, int32_t world, int32_t tiles_cap, int32_t tiles,
                     int32_t batch, void* residual, int64_t residual_stride,
                     const void* norm_weight, float eps, void* out, int64_t out_stride,
                     int32_t payload, void* stream) {
  PG_REQUIRE(exchange != nullptr && aligned(exchange, 256), "the exchange buffer is required");
  PG_REQUIRE(payload == PG_TP_PAYLOAD_F32 || payload == PG_TP_PAYLOAD_F16,
             "payload must be PG_TP_PAYLOAD_F32 (a publishing pg_skinny_gemm) or "
             "PG_TP_PAYLOAD_F16 (pg_tp_publish)");
  PG_REQUIRE(world >= 2 && world <= pg::kGemmMaxTp, "world must be 2..8");
  PG_REQUIRE(tiles >= 1 && tiles <= tiles_cap && tiles * pg::kGemmTileRows <= 16384,
             "tiles must be 1..tiles_cap with at most 16384 columns");
  PG_REQUIRE(batch >= 1 && batch <= pg::kGemmMaxXR, "batch must be 1..32");
  PG_REQUIRE(out != nullptr && aligned(out, 16) && out_stride % 8 == 0,
             "out must be 16-byte aligned with rows of 8k halves");
  if (residual != nullptr)
    PG_REQUIRE(aligned(residual, 16) && residual_stride % 8 == 0,
               "residual must be 16-byte aligned with rows of 8k halves");
  if (norm_weight != nullptr) {
    PG_REQUIRE(residual != nullptr, "the RMSNorm applies to the updated residual");
    PG_REQUIRE(aligned(norm_weight, 16) && eps > 0.f, "norm weight / eps invalid");
  }
  pg::TpReduceParams p{};
  p.exchange = static_cast<const uint8_t*>(exchange);
  p.world = world;
  p.cap = tiles_cap;
  p.tiles = tiles;
  p.residual = static_cast<__half*>(residual);
  p.residual_stride = residual_stride;
  p.norm_w = static_cast<const __half*>(norm_weight);
  p.eps = eps;
  p.out = static_cast<__half*>(out);
  p.out_stride = out_stride;
  p.error_flag = device_error_ptr();
  if (payload == PG_TP_PAYLOAD_F16)
    return launch_pdl(pg::pg_tp_reduce_kernel<true>, dim3(batch), dim3(pg::kTpReduceThreads), 0,
                      static_cast<cudaStream_t>(stream), "tp reduce launch", p);
  return launch_pdl(pg::pg_tp_reduce_kernel<false>, dim3(batch), dim3(pg::kTpReduceThreads), 0,
                    static_cast<cudaStream_t>(stream), "tp reduce launch", p);
}

// --------------------------------------------- allocation-free decode
// Some callers cannot allocate device memory: a plugin loaded into a host
// process whose allocator owns the device (or forbids allocation while it
// runs), or code that must not allocate inside a latency-critical path.
// pg_decode_static gives them the planned split decode + merge with its
// scratch (work list, per-head item ranges, split partial states) in this
// file-scope device array instead of a caller workspace.  Every GPU that
// loads the library holds the array until the process exits.
constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
constexpr int64_t kStaticMaxItems = 4096;
constexpr int64_t kStaticMaxHeads = 8192;  // batch * kv_heads
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {
std::mutex g_static_mu;
unsigned char* g_static_dev[64] = {nullptr};  // device address, per device
// Host staging of the plan (no heap allocation on the call path).
pg_decode_item g_static_items[kStaticMaxItems];
int32_t g_static_off[kStaticMaxHeads + 1];

size_t align256(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

int32_t pg_decode_static(const pg_decode_args* args, const int32_t* indptr0,
                         const int32_t* indptr1, int32_t split_pages0,
                         int32_t split_pages1, int32_t num_sms, void* stream) {
  PG_REQUIRE(args != nullptr, "null arguments");
  {
    // Every call copies its plan from host memory, which a stream capture
    // cannot record; refuse before enqueuing anything, so the caller's
    // capture stays valid.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    int32_t rc0 = cuda_check(cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cs),
                             "cudaStreamIsCapturing");
    if (rc0 != PG_OK) return rc0;
    PG_REQUIRE(cs == cudaStreamCaptureStatusNone,
               "pg_decode_static cannot run while its stream is being captured: it copies "
               "its plan from host memory on every call");
  }
  PG_REQUIRE(static_cast<int64_t>(args->batch) * args->kv_heads <= kStaticMaxHeads,
             "pg_decode_static supports at most %lld (request, kv head) pairs",
             static_cast<long long>(kStaticMaxHeads));
  std::lock_guard<std::mutex> lock(g_static_mu);
  int dev = 0;
  int32_t rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != PG_OK) return rc;
  PG_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range");
  if (g_static_dev[dev] == nullptr) {
    // One-time set-up per device, with that device current: the symbol's
    // device address (the host-side name is only a stand-in).
    void* ptr = nullptr;
    rc = cuda_check(cudaGetSymbolAddress(&ptr, g_static_scratch),
                    "cudaGetSymbolAddress(static decode scratch)");
    if (rc != PG_OK) return rc;
    g_static_dev[dev] = static_cast<unsigned char*>(ptr);
  }
  unsigned char* base = g_static_dev[dev];
  pg_plan_info info{};
  rc = pg_decode_plan(args->batch, args->kv_heads, indptr0, indptr1, split_pages0,
                      split_pages1, num_sms, args->warps_per_cta, g_static_items,
                      kStaticMaxItems, g_static_off, &info);
  if (rc == PG_ERR_CAPACITY)
    return fail(PG_ERR_CAPACITY,
                "pg_decode_static: the plan needs %lld work items; the static scratch holds at "
                "most %lld (use a larger split)",
                static_cast<long long>(info.num_items), static_cast<long long>(kStaticMaxItems));
  if (rc != PG_OK) return rc;
  const int64_t n = info.num_items;
  const int64_t heads = static_cast<int64_t>(args->batch) * args->kv_heads;
  const size_t items_b = align256(static_cast<size_t>(kStaticMaxItems) * sizeof(pg_decode_item));
  const size_t off_b = align256(static_cast<size_t>(kStaticMaxHeads + 1) * sizeof(int32_t));
  const size_t lse_b = align256(static_cast<size_t>(n) * args->group * sizeof(float));
  const size_t o_b = static_cast<size_t>(n) * args->group * pg::kHeadDim * sizeof(float);
  if (items_b + off_b + lse_b + o_b > kStaticScratchBytes)
    return fail(PG_ERR_CAPACITY,
                "pg_decode_static: %lld work items need %zu bytes of scratch; the static array "
                "holds %zu (use a larger split)",
                static_cast<long long>(n), items_b + off_b + lse_b + o_b, kStaticScratchBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Pageable host -> device copies are staged before returning, so the host
  // plan buffers may be rewritten by the next call right away.
  if (n > 0) {
    rc = cuda_check(cudaMemcpyAsync(base, g_static_items, static_cast<size_t>(n) * sizeof(pg_decode_item),
                                    cudaMemcpyHostToDevice, st),
                    "copy work items");
    if (rc != PG_OK) return rc;
  }
  rc = cuda_check(cudaMemcpyAsync(base + items_b, g_static_off, static_cast<size_t>(heads + 1) * sizeof(int32_t),
                                  cudaMemcpyHostToDevice, st),
                  "copy item offsets");
  if (rc != PG_OK) return rc;
  pg_decode_args a = *args;
  a.items = reinterpret_cast<const pg_decode_item*>(base);
  a.item_off = reinterpret_cast<const int32_t*>(base + items_b);
  a.num_items = static_cast<int32_t>(n);
  a.warps_per_cta = info.warps_per_cta;
  a.part_lse = reinterpret_cast<float*>(base + items_b + off_b);
  a.part_o = reinterpret_cast<float*>(base + items_b + off_b + lse_b);
  a.final_mode = info.single_item_per_head;
  a.merge_sem = nullptr;  // separate merge launch: nothing has to start at zero
  a.stage_mask = 0;
  return pg_decode_run(&a, stream);
}

}  // extern "C"
