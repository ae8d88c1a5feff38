// spd_abi.cu — the extern "C" boundary of libspd_b200.so.
//
// Every entry point validates its arguments on the host, records a readable message
// for spd_get_last_error() on failure, and enqueues kernels on the caller's stream.
// Nothing here allocates device memory, synchronises, or reads device values (except
// spd_read_error_word, which exists to do exactly that outside graph capture).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "spd_params.cuh"

namespace spd {
int paged_decode_attn_launch(const PagedParams& p, int dtype, int D, int bs, int sms, cudaStream_t st);
int cross_attn_launch(const CrossParams& p, int dtype, int D, int sms, cudaStream_t st);
int kv_append_launch(const AppendParams& p, int sms, cudaStream_t st);
int block_gather_launch(const GatherParams& p, int sms, cudaStream_t st);
int add_layernorm_launch(const AddLnParams& p, int dtype, cudaStream_t st);
int argmax_rows_launch(const ArgmaxParams& p, int dtype, cudaStream_t st);
int linear_small_m_launch(const void* x, const void* w, const void* bias, void* y, int M, int N, int K,
                          long long group_cols, long long group_stride, int act, int dtype, int* err, int sms,
                          cudaStream_t st);
int cross_kv_project_launch(const void* enc_out, const void* w_kv, const void* b_kv, void* out,
                            const int32_t* slot_ids, int B, int T, int d_model, int L, int H, int D,
                            int T_out, int64_t out_slot_stride, int dtype, int* err, int sms, cudaStream_t st);
}  // namespace spd

namespace {

thread_local char g_err_msg[512] = {0};
thread_local int g_err_code = SPD_OK;
// Bound on the attention kernels' waits for launches made by this thread.
thread_local unsigned long long g_wait_ns = spd::SPD_WAIT_NS;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err_msg, sizeof(g_err_msg), fmt, ap);
  va_end(ap);
  g_err_code = code;
  return code;
}

int ok() {
  g_err_code = SPD_OK;
  g_err_msg[0] = 0;
  return SPD_OK;
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case SPD_F32: return 4;
    case SPD_F16: return 2;
    case SPD_BF16: return 2;
    default: return 0;
  }
}

// SM count per device, cached (the device list does not change under a process).
int sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0) {
    if (cudaGetDevice(&device) != cudaSuccess) return 0;
  }
  if (device >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device] = n;
  }
  return cache[device];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool head_dim_ok(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

}  // namespace

namespace spd {
// Records a host-side error for spd_get_last_error() from other translation units of
// the library; returns `code`.
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }

// Host-side argument checks of spd_paged_decode_attn (everything but the workspace), shared
// with the allocation-free entry point, which must refuse a call before touching its scratch.
int paged_decode_attn_check(const void* q, const void* k_pool, const void* v_pool, const int32_t* block_tables,
                            const int32_t* context_lens, const void* out, int B, int H, int D, int block_size,
                            int max_blocks, int num_blocks, int dtype, const void* k_new, const void* v_new) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_paged_decode_attn: dtype %d not supported", dtype);
  if (!q || !k_pool || !v_pool || !block_tables || !context_lens || !out)
    return fail(SPD_ERR_INVALID_ARG, "spd_paged_decode_attn: null tensor pointer");
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(SPD_ERR_INVALID_ARG, "spd_paged_decode_attn: k_new and v_new must both be given or both NULL");
  if (B <= 0 || B > 4096 || H <= 0 || H > 32 || max_blocks <= 0 || num_blocks <= 0)
    return fail(SPD_ERR_INVALID_ARG, "spd_paged_decode_attn: bad sizes B=%d H=%d max_blocks=%d num_blocks=%d",
                B, H, max_blocks, num_blocks);
  if (!head_dim_ok(D)) return fail(SPD_ERR_UNSUPPORTED, "spd_paged_decode_attn: head_dim %d not supported", D);
  if (block_size != 8 && block_size != 16 && block_size != 32)
    return fail(SPD_ERR_UNSUPPORTED, "spd_paged_decode_attn: block_size %d not supported", block_size);
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out) ||
      (k_new && (!aligned16(k_new) || !aligned16(v_new))))
    return fail(SPD_ERR_INVALID_ARG, "spd_paged_decode_attn: tensors must be 16-byte aligned");
  return SPD_OK;
}
}  // namespace spd

namespace {
// An mbarrier phase that never completes (it expects 16 bytes that no copy delivers):
// the bounded wait must give up after limit_ns, record SPD_DEVERR_TIMEOUT and return.
// No asynchronous operation is ever issued, so the CTA exits with nothing in flight.
__global__ void wait_timeout_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    spd::mbar_init(&bar, 1);
    spd::fence_barrier_init();
    spd::mbar_arrive_expect_tx(&bar, 16);
    (void)spd::mbar_wait_bounded(&bar, 0, err, limit_ns);
  }
}
}  // namespace

extern "C" {

int spd_version(void) { return 100; }

int spd_set_wait_timeout_ns(uint64_t ns) {
  g_wait_ns = ns ? (unsigned long long)ns : spd::SPD_WAIT_NS;
  return ok();
}

uint64_t spd_get_wait_timeout_ns(void) { return g_wait_ns; }

int spd_selftest_wait_timeout(int32_t* error_word, uint64_t timeout_ns, void* stream) {
  if (!error_word || timeout_ns == 0 || timeout_ns > spd::SPD_WAIT_NS)
    return fail(SPD_ERR_INVALID_ARG, "spd_selftest_wait_timeout: error_word and 0 < timeout_ns <= %llu needed",
                (unsigned long long)spd::SPD_WAIT_NS);
  wait_timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<int*>(error_word),
                                                                            (unsigned long long)timeout_ns);
  if (cudaGetLastError() != cudaSuccess) return fail(SPD_ERR_CUDA, "spd_selftest_wait_timeout: launch failed");
  return ok();
}

int spd_get_last_error(char* buf, size_t size) {
  if (buf && size) {
    strncpy(buf, g_err_msg, size - 1);
    buf[size - 1] = 0;
  }
  return g_err_code;
}

size_t spd_paged_decode_attn_workspace_size(int B, int H, int D, int max_blocks, int device) {
  if (B <= 0 || H <= 0 || D <= 0 || max_blocks <= 0 || sm_count(device) <= 0) return 0;
  const size_t items = (size_t)B * ((max_blocks + spd::kItemUnits - 1) / spd::kItemUnits);
  return spd::kWsHeaderBytes + spd::round_up((size_t)B * H * 4, 256) +
         spd::round_up(items * H * (D + 8) * 4, 256);  // partial rows of D + 8 floats
}

size_t spd_cross_attn_workspace_size(int B, int H, int D, int device) {
  if (B <= 0 || H <= 0 || D <= 0 || sm_count(device) <= 0) return 0;
  return spd::kWsHeaderBytes + spd::round_up((size_t)B * H * 4, 256) +
         spd::round_up((size_t)B * H * spd::kCrossMaxItems * (D + 2) * 4, 256);  // a partial row per item
}

int spd_read_error_word(const void* error_word, int32_t* host_word, void* stream) {
  if (!error_word || !host_word) return fail(SPD_ERR_INVALID_ARG, "spd_read_error_word: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_word, error_word, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(SPD_ERR_CUDA, "spd_read_error_word: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_paged_decode_attn(const void* q, void* k_pool, void* v_pool, const int32_t* block_tables,
                          const int32_t* context_lens, void* out, int B, int H, int D, int block_size,
                          int max_blocks, int num_blocks, float scale, int dtype, const void* k_new,
                          const void* v_new, void* workspace, size_t workspace_bytes, void* stream) {
  const int rc0 = spd::paged_decode_attn_check(q, k_pool, v_pool, block_tables, context_lens, out, B, H, D,
                                               block_size, max_blocks, num_blocks, dtype, k_new, v_new);
  if (rc0 != SPD_OK) return rc0;
  const size_t need = spd_paged_decode_attn_workspace_size(B, H, D, max_blocks, -1);
  if (!workspace || workspace_bytes < need)
    return fail(SPD_ERR_WORKSPACE, "spd_paged_decode_attn: workspace %zu bytes, need %zu", workspace_bytes, need);
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_paged_decode_attn: no CUDA device");

  spd::PagedParams p{};
  p.q = q; p.k_pool = k_pool; p.v_pool = v_pool; p.block_tables = block_tables;
  p.context_lens = context_lens; p.out = out; p.k_new = k_new; p.v_new = v_new;
  p.B = B; p.H = H; p.max_blocks = max_blocks; p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_ns = g_wait_ns;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.err = reinterpret_cast<int*>(ws);
  p.work = reinterpret_cast<int*>(ws + spd::kWsWorkOffset);
  p.counters = reinterpret_cast<int*>(ws + spd::kWsHeaderBytes);
  p.partials = reinterpret_cast<float*>(ws + spd::kWsHeaderBytes + spd::round_up((size_t)B * H * 4, 256));
  const int rc = spd::paged_decode_attn_launch(p, dtype, D, block_size, sms, static_cast<cudaStream_t>(stream));
  if (rc == SPD_ERR_UNSUPPORTED)
    return fail(rc, "spd_paged_decode_attn: H=%d D=%d block_size=%d dtype=%d does not fit shared memory", H, D,
                block_size, dtype);
  if (rc != SPD_OK) return fail(rc, "spd_paged_decode_attn: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_cross_attn(const void* q, const void* k, const void* v, const int32_t* valid_lens, void* out, int B, int H,
                   int D, int T_max, int64_t kv_batch_stride, int64_t kv_head_stride, float scale, int dtype,
                   void* workspace, size_t workspace_bytes, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_cross_attn: dtype %d not supported", dtype);
  if (!q || !k || !v || !valid_lens || !out) return fail(SPD_ERR_INVALID_ARG, "spd_cross_attn: null tensor pointer");
  if (B <= 0 || B > 4096 || H <= 0 || (long long)B * H > 65536 || T_max <= 0)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_attn: bad sizes B=%d H=%d T_max=%d", B, H, T_max);
  if (!head_dim_ok(D)) return fail(SPD_ERR_UNSUPPORTED, "spd_cross_attn: head_dim %d not supported", D);
  if (kv_head_stride < (int64_t)T_max * D || kv_batch_stride < 0)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_attn: kv_head_stride %lld < T_max*D", (long long)kv_head_stride);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (kv_batch_stride * eb) % 16 ||
      (kv_head_stride * eb) % 16)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_attn: pointers and strides must be 16-byte aligned");
  const size_t need = spd_cross_attn_workspace_size(B, H, D, -1);
  if (!workspace || workspace_bytes < need)
    return fail(SPD_ERR_WORKSPACE, "spd_cross_attn: workspace %zu bytes, need %zu", workspace_bytes, need);
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_cross_attn: no CUDA device");

  spd::CrossParams p{};
  p.q = q; p.k = k; p.v = v; p.valid_lens = valid_lens; p.out = out;
  p.B = B; p.H = H; p.T_max = T_max;
  p.kv_batch_stride = kv_batch_stride; p.kv_head_stride = kv_head_stride;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_ns = g_wait_ns;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.err = reinterpret_cast<int*>(ws);
  p.work = reinterpret_cast<int*>(ws + spd::kWsWorkOffset);
  p.partials = reinterpret_cast<float*>(ws + spd::kWsHeaderBytes + spd::round_up((size_t)B * H * 4, 256));
  const int rc = spd::cross_attn_launch(p, dtype, D, sms, static_cast<cudaStream_t>(stream));
  if (rc != SPD_OK) return fail(rc, "spd_cross_attn: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_kv_append(const void* k_src, const void* v_src, int64_t src_stride_b, int64_t src_stride_h,
                  int64_t src_stride_t, void* k_pool, void* v_pool, const int32_t* block_tables,
                  const int32_t* positions, int B, int T, int H, int D, int block_size, int max_blocks,
                  int num_blocks, int dtype, int32_t* error_word, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_kv_append: dtype %d not supported", dtype);
  if (!k_src || !k_pool || !block_tables || !positions)
    return fail(SPD_ERR_INVALID_ARG, "spd_kv_append: null tensor pointer");
  if ((v_src == nullptr) != (v_pool == nullptr))
    return fail(SPD_ERR_INVALID_ARG, "spd_kv_append: v_src and v_pool must both be given or both NULL");
  if (B < 0 || T < 0 || H <= 0 || D <= 0 || block_size <= 0 || max_blocks <= 0 || num_blocks <= 0)
    return fail(SPD_ERR_INVALID_ARG, "spd_kv_append: bad sizes");
  if ((D * eb) % 2) return fail(SPD_ERR_INVALID_ARG, "spd_kv_append: row bytes must be even");
  if (!aligned16(k_pool) || (v_pool && !aligned16(v_pool)))
    return fail(SPD_ERR_INVALID_ARG, "spd_kv_append: pools must be 16-byte aligned");
  if (B == 0 || T == 0) return ok();
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_kv_append: no CUDA device");
  spd::AppendParams p{};
  p.k_src = static_cast<const unsigned char*>(k_src);
  p.v_src = static_cast<const unsigned char*>(v_src);
  p.sb = src_stride_b * eb; p.sh = src_stride_h * eb; p.st = src_stride_t * eb;
  p.k_pool = static_cast<unsigned char*>(k_pool);
  p.v_pool = static_cast<unsigned char*>(v_pool);
  p.block_tables = block_tables; p.positions = positions;
  p.B = B; p.T = T; p.H = H; p.row_bytes = D * eb; p.block_size = block_size;
  p.max_blocks = max_blocks; p.num_blocks = num_blocks; p.err = error_word;
  const int rc = spd::kv_append_launch(p, sms, static_cast<cudaStream_t>(stream));
  if (rc != SPD_OK) return fail(rc, "spd_kv_append: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_block_gather(const void* pool, const int32_t* block_tables, const int32_t* seq_lens, void* out, int B,
                     int H, int D, int block_size, int max_blocks, int num_blocks, int T_out,
                     int64_t out_batch_stride, int zero_pad, int dtype, int32_t* error_word, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_block_gather: dtype %d not supported", dtype);
  if (!pool || !block_tables || !seq_lens || !out) return fail(SPD_ERR_INVALID_ARG, "spd_block_gather: null pointer");
  if (B < 0 || H <= 0 || D <= 0 || block_size <= 0 || max_blocks <= 0 || num_blocks <= 0 || T_out < 0)
    return fail(SPD_ERR_INVALID_ARG, "spd_block_gather: bad sizes");
  if ((D * eb) % 16 || !aligned16(pool) || !aligned16(out) || (out_batch_stride * eb) % 16)
    return fail(SPD_ERR_INVALID_ARG, "spd_block_gather: rows, pointers and strides must be 16-byte aligned");
  if (out_batch_stride < (int64_t)H * T_out * D && B > 1)
    return fail(SPD_ERR_INVALID_ARG, "spd_block_gather: out_batch_stride smaller than H*T_out*D");
  if (B == 0 || T_out == 0) return ok();
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_block_gather: no CUDA device");
  spd::GatherParams p{};
  p.pool = static_cast<const unsigned char*>(pool);
  p.block_tables = block_tables; p.seq_lens = seq_lens;
  p.out = static_cast<unsigned char*>(out);
  p.B = B; p.H = H; p.row_bytes = D * eb; p.block_size = block_size; p.max_blocks = max_blocks;
  p.num_blocks = num_blocks; p.T_out = T_out; p.zero_pad = zero_pad;
  p.out_batch_stride = out_batch_stride * eb; p.err = error_word;
  const int rc = spd::block_gather_launch(p, sms, static_cast<cudaStream_t>(stream));
  if (rc != SPD_OK) return fail(rc, "spd_block_gather: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_add_layernorm(const void* x, const void* delta, const void* gamma, const void* beta, void* x_out, void* y,
                      int rows, int cols, int64_t y_ld, float eps, int dtype, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_add_layernorm: dtype %d not supported", dtype);
  if (!x || !gamma || !beta || !y || (delta && !x_out)) return fail(SPD_ERR_INVALID_ARG, "spd_add_layernorm: null pointer");
  if (rows < 0 || cols <= 0) return fail(SPD_ERR_INVALID_ARG, "spd_add_layernorm: bad sizes");
  if ((cols * eb) % 16 || !aligned16(x) || !aligned16(gamma) || !aligned16(beta) || !aligned16(y) ||
      (delta && (!aligned16(delta) || !aligned16(x_out))))
    return fail(SPD_ERR_INVALID_ARG, "spd_add_layernorm: rows and pointers must be 16-byte aligned");
  if (cols > 2048) return fail(SPD_ERR_UNSUPPORTED, "spd_add_layernorm: rows of at most 2048 elements");
  if (y_ld == 0) y_ld = cols;
  if (y_ld < cols || (y_ld * eb) % 16)
    return fail(SPD_ERR_INVALID_ARG, "spd_add_layernorm: y_ld %lld must be >= cols and a multiple of 16 bytes",
                (long long)y_ld);
  if (rows == 0) return ok();
  spd::AddLnParams p{x, delta, gamma, beta, x_out, y, rows, cols, (long long)y_ld, eps};
  const int rc = spd::add_layernorm_launch(p, dtype, static_cast<cudaStream_t>(stream));
  if (rc == SPD_ERR_UNSUPPORTED) return fail(rc, "spd_add_layernorm: row length not supported");
  if (rc != SPD_OK) return fail(rc, "spd_add_layernorm: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_argmax_rows(const void* x, int rows, int cols, int64_t ld, const void* skip_mask, int64_t* out, int dtype,
                    void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(SPD_ERR_UNSUPPORTED, "spd_argmax_rows: dtype %d not supported", dtype);
  if (!x || !out) return fail(SPD_ERR_INVALID_ARG, "spd_argmax_rows: null pointer");
  if (rows < 0 || cols <= 0 || ld < cols) return fail(SPD_ERR_INVALID_ARG, "spd_argmax_rows: bad sizes");
  if (rows == 0) return ok();
  spd::ArgmaxParams p{x, skip_mask, reinterpret_cast<long long*>(out), rows, cols, (long long)ld,
                      (aligned16(x) && (ld * eb) % 16 == 0) ? 1 : 0};
  const int rc = spd::argmax_rows_launch(p, dtype, static_cast<cudaStream_t>(stream));
  if (rc != SPD_OK) return fail(rc, "spd_argmax_rows: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_linear(const void* x, const void* w, const void* bias, void* y, int M, int N, int K, int64_t y_group_cols,
               int64_t y_group_stride, int activation, int dtype, int32_t* error_word, void* stream) {
  if (dtype != SPD_F16 && dtype != SPD_BF16)
    return fail(SPD_ERR_UNSUPPORTED, "spd_linear: dtype %d not supported (F16/BF16 only)", dtype);
  if (!x || !w || !y) return fail(SPD_ERR_INVALID_ARG, "spd_linear: null pointer");
  if (M < 1 || M > 64 || N < 1 || K < 64 || K % 64)
    return fail(SPD_ERR_UNSUPPORTED, "spd_linear: need 1 <= M <= 64 and K a multiple of 64 (M=%d N=%d K=%d)", M, N,
                K);
  if (y_group_cols <= 0) y_group_cols = N;
  if (N % y_group_cols || (N > y_group_cols && y_group_stride < (int64_t)M * y_group_cols))
    return fail(SPD_ERR_INVALID_ARG, "spd_linear: N must be a multiple of y_group_cols, planes must not overlap");
  if (activation != SPD_ACT_NONE && activation != SPD_ACT_GELU)
    return fail(SPD_ERR_INVALID_ARG, "spd_linear: unknown activation %d", activation);
  if (!aligned16(x) || !aligned16(w) || (reinterpret_cast<uintptr_t>(y) & 1) ||
      (bias && (reinterpret_cast<uintptr_t>(bias) & 1)))
    return fail(SPD_ERR_INVALID_ARG, "spd_linear: x and w must be 16-byte aligned");
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_linear: no CUDA device");
  const int rc = spd::linear_small_m_launch(x, w, bias, y, M, N, K, y_group_cols, y_group_stride, activation, dtype,
                                            error_word, sms, static_cast<cudaStream_t>(stream));
  if (rc != SPD_OK) return fail(rc, "spd_linear: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

int spd_cross_kv_project(const void* enc_out, const void* w_kv, const void* b_kv, void* out,
                         const int32_t* slot_ids, int B, int T, int d_model, int L, int H, int D, int T_out,
                         int64_t out_slot_stride, int dtype, int32_t* error_word, void* stream) {
  if (dtype != SPD_F16 && dtype != SPD_BF16)
    return fail(SPD_ERR_UNSUPPORTED, "spd_cross_kv_project: dtype %d not supported (F16/BF16 only)", dtype);
  if (!enc_out || !w_kv || !out) return fail(SPD_ERR_INVALID_ARG, "spd_cross_kv_project: null pointer");
  if (B <= 0 || T <= 0 || d_model <= 0 || L <= 0 || H <= 0 || D <= 0 || T_out < T)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_kv_project: bad sizes");
  if (d_model % 64 || D % 8)
    return fail(SPD_ERR_UNSUPPORTED, "spd_cross_kv_project: need d_model %% 64 == 0 and D %% 8 == 0");
  if (!aligned16(enc_out) || !aligned16(w_kv) || !aligned16(out) || (b_kv && !aligned16(b_kv)) ||
      (out_slot_stride * 2) % 16)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_kv_project: pointers and strides must be 16-byte aligned");
  if (out_slot_stride < (int64_t)L * 2 * H * T_out * D)
    return fail(SPD_ERR_INVALID_ARG, "spd_cross_kv_project: out_slot_stride smaller than L*2*H*T_out*D");
  const int sms = sm_count(-1);
  if (sms <= 0) return fail(SPD_ERR_CUDA, "spd_cross_kv_project: no CUDA device");
  const int rc = spd::cross_kv_project_launch(enc_out, w_kv, b_kv, out, slot_ids, B, T, d_model, L, H, D, T_out,
                                              out_slot_stride, dtype, error_word, sms,
                                              static_cast<cudaStream_t>(stream));
  if (rc == SPD_ERR_UNSUPPORTED) return fail(rc, "spd_cross_kv_project: shape not supported");
  if (rc != SPD_OK) return fail(rc, "spd_cross_kv_project: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

}  // extern "C"
