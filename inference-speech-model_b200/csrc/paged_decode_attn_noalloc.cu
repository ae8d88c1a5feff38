// paged_decode_attn_noalloc.cu — spd_paged_decode_attn for callers that cannot allocate.
//
// Some hosts of this library may not call cudaMalloc at all (allocator callbacks, plugin
// frameworks that pass in only the call's tensors, fixed-budget processes), so they
// cannot provide the workspace spd_paged_decode_attn needs for its split-KV counters and
// partial results.  This entry point keeps that scratch in a file-scope device array of
// SPD_NOALLOC_SCRATCH_BYTES instead.  In host code `g_noalloc_scratch` only names the
// symbol — it is not a device address — so each device's address is looked up once with
// cudaGetSymbolAddress (with that device current) and cached for the life of the process
// (a cudaDeviceReset invalidates the cached address; calls after one are not supported).
#include <cstdio>
#include <mutex>

#include "spd_params.cuh"

namespace spd {
int record_error(int code, const char* msg);
int paged_decode_attn_check(const void* q, const void* k_pool, const void* v_pool, const int32_t* block_tables,
                            const int32_t* context_lens, const void* out, int B, int H, int D, int block_size,
                            int max_blocks, int num_blocks, int dtype, const void* k_new, const void* v_new);
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[SPD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up on first use).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return spd::record_error(SPD_ERR_CUDA, "spd_paged_decode_attn_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (rc != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof(msg), "spd_paged_decode_attn_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(rc));
      return spd::record_error(SPD_ERR_CUDA, msg);
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SPD_OK;
}

// ORs this call's device error flags (the scratch header's word) into the caller's word,
// which may carry flags from earlier calls or other ops.
__global__ void or_error_word(int32_t* dst, const int32_t* src) {
  const int32_t v = *src;
  if (v) atomicOr(dst, v);
}

}  // namespace

extern "C" int spd_paged_decode_attn_noalloc(const void* q, void* k_pool, void* v_pool,
                                             const int32_t* block_tables, const int32_t* context_lens,
                                             void* out, int B, int H, int D, int block_size, int max_blocks,
                                             int num_blocks, float scale, int dtype, const void* k_new,
                                             const void* v_new, int32_t* error_word, void* stream) {
  // every argument check comes before the shared scratch is touched: a refused call must
  // not clear counters that a call still running on the GPU is using
  int rc = spd::paged_decode_attn_check(q, k_pool, v_pool, block_tables, context_lens, out, B, H, D, block_size,
                                        max_blocks, num_blocks, dtype, k_new, v_new);
  if (rc != SPD_OK) return rc;
  const size_t need = spd_paged_decode_attn_workspace_size(B, H, D, max_blocks, -1);
  if (need == 0) return spd::record_error(SPD_ERR_CUDA, "spd_paged_decode_attn_noalloc: no CUDA device");
  if (need > SPD_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "spd_paged_decode_attn_noalloc: B=%d H=%d D=%d max_blocks=%d needs %zu bytes of scratch, more "
             "than the %u-byte array; use spd_paged_decode_attn with a workspace",
             B, H, D, max_blocks, need, (unsigned)SPD_NOALLOC_SCRATCH_BYTES);
    return spd::record_error(SPD_ERR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  rc = scratch_for_current_device(&scratch);
  if (rc != SPD_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The header (error word, work counters) and the arrival counters must start at zero;
  // the previous call may have used another geometry, which moves where they sit.
  const size_t clear = spd::kWsHeaderBytes + spd::round_up((size_t)B * H * 4, 256);
  if (cudaMemsetAsync(scratch, 0, clear, st) != cudaSuccess)
    return spd::record_error(SPD_ERR_CUDA, "spd_paged_decode_attn_noalloc: clearing the scratch counters failed");
  rc = spd_paged_decode_attn(q, k_pool, v_pool, block_tables, context_lens, out, B, H, D, block_size, max_blocks,
                             num_blocks, scale, dtype, k_new, v_new, scratch, SPD_NOALLOC_SCRATCH_BYTES, stream);
  if (rc != SPD_OK) return rc;  // the message is already recorded
  if (error_word) {
    or_error_word<<<1, 1, 0, st>>>(error_word, static_cast<const int32_t*>(scratch));
    if (cudaGetLastError() != cudaSuccess)
      return spd::record_error(SPD_ERR_CUDA, "spd_paged_decode_attn_noalloc: passing on the error word failed");
  }
  return SPD_OK;
}
