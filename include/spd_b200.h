/*
 * spd_b200.h — C ABI of the B200 (sm_100a) speech-decode hot path.
 *
 * One shared library (libspd_b200.so) exports the five decode-path operations of the
 * Whisper-class serving engine plus error/workspace helpers.  Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t passed as `void*`
 *     (NULL = legacy default stream); no torch types cross this boundary;
 *   - returns an int status (SPD_OK == 0); on failure spd_get_last_error() gives text;
 *   - allocates nothing, synchronises nothing and reads no device value on the host,
 *     so every call can be captured into a CUDA graph;
 *   - validates arguments on the host (SPD_ERR_INVALID_ARG / SPD_ERR_UNSUPPORTED);
 *     out-of-range block ids or lengths found on the device are clamped to in-bounds
 *     addresses and recorded in a device error word (see SPD_DEVERR_*), never trapped.
 *
 * Pool layout (decoder paged KV cache and encoder paged pool), one tensor per layer and
 * per K/V:  pool[num_blocks][block_size][H][D], element type given by `dtype`.
 * Block tables are int32 [B][max_blocks]; lengths / positions are int32 [B].
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   spd_paged_decode_attn  scripts/evaluate_paging_variants.py:56-133 (Triton
 *                          paged_decode_attention_kernel, launched at :632-642) and the
 *                          decoder self-attention math of speech_serving/models.py:126-165,
 *                          :443-466 (graph step: scatter + masked full-bucket attention)
 *   spd_cross_attn         speech_serving/models.py:167-203 (eager cross-attention) and
 *                          :468-479 (graph step over g_cross_kv with additive mask)
 *   spd_kv_append          speech_serving/phase_aware_scheduler.py:1004-1010 (per-token
 *                          paged write), :678-690 (prompt K/V block writes),
 *                          speech_serving/models.py:449-454 and
 *                          speech_serving/graph_decode_buffers.py:56-59 (scatter_ at position),
 *                          speech_serving/encoder_block_manager.py:177-192 (store_encoder_kv)
 *   spd_block_gather       speech_serving/phase_aware_scheduler.py:613-624, :859-882,
 *                          :926-962 and speech_serving/encoder_attention.py:50-63
 *                          (pool[table].view(-1,H,D)[:T].permute(1,0,2), zero padded)
 *   spd_cross_kv_project   speech_serving/models.py:554-561 (per-decoder-layer
 *                          encoder_attn.k_proj / v_proj over the encoder output)
 *   spd_add_layernorm      the residual add and the LayerNorm after it in every decoder
 *                          layer, speech_serving/models.py:163-207 (x = residual + ...;
 *                          norm2 / norm3), and transformers' WhisperDecoderLayer
 *   spd_argmax_rows        the greedy pick after the output projection:
 *                          speech_serving/graph_decode_buffers.py:446-448 (suppress mask,
 *                          argmax) and speech_serving/models.py:487
 *   spd_linear             the decode step's Linear layers: speech_serving/models.py:127-129
 *                          (q/k/v), :159 (self out), :178-180 (cross q), :202 (cross out),
 *                          :205-207 (MLP with GELU), :487 (lm_head), and the same layers of
 *                          transformers' WhisperDecoderLayer / proj_out (models.py:593-603)
 */
#ifndef SPD_B200_H
#define SPD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define SPD_OK 0
#define SPD_ERR_INVALID_ARG 1   /* bad pointer / size / alignment */
#define SPD_ERR_UNSUPPORTED 2   /* shape or dtype combination not compiled */
#define SPD_ERR_CUDA 3          /* a CUDA runtime call failed (launch, attribute) */
#define SPD_ERR_WORKSPACE 4     /* workspace missing or smaller than *_workspace_size() */

/* ---- element types --------------------------------------------------------------- */
#define SPD_F32 0
#define SPD_F16 1
#define SPD_BF16 2

/* ---- device error word codes (bit flags, OR-ed into workspace/error word) -------- */
#define SPD_DEVERR_BLOCK_ID 1      /* block table entry outside [0, num_blocks) */
#define SPD_DEVERR_LENGTH 2        /* length / position beyond max_blocks*block_size or T_max */
#define SPD_DEVERR_TIMEOUT 4       /* a bounded wait on an async copy ran out */

/* Library version (major*100 + minor). */
int spd_version(void);

/* Copies the last host-side error message of this thread into buf (NUL-terminated).
 * Returns the status code that produced it (SPD_OK if none). */
int spd_get_last_error(char* buf, size_t size);

/* Number of bytes of workspace the attention kernels need.  The workspace holds a
 * 256-byte header (device error word at offset 0, work counters), arrival counters and
 * fp32 split-KV partial results.  It must be zero-filled once before first use; the
 * kernels leave every counter back at zero, so it can be reused by later calls with the
 * same geometry on the same stream.  A workspace used with another geometry must be
 * zero-filled again first; calls that overlap on the GPU must use separate workspaces.
 * `device` < 0 means the current device. */
size_t spd_paged_decode_attn_workspace_size(int B, int H, int D, int max_blocks, int device);
size_t spd_cross_attn_workspace_size(int B, int H, int D, int device);

/* Bound on every wait of the attention kernels (spd_paged_decode_attn, its allocation-free
 * variant, spd_cross_attn) launched by the calling thread from now on; each launch takes
 * the value as a kernel parameter.  A wait that runs out records SPD_DEVERR_TIMEOUT in the
 * error word, the launch stops its work (outputs are then undefined), waits for its own
 * copies in flight and returns; the context stays usable.  0 restores the default of 2 s
 * (SPD_DEFAULT_WAIT_NS).  No counterpart in the reference, whose kernels never wait. */
#define SPD_DEFAULT_WAIT_NS 2000000000ull
int spd_set_wait_timeout_ns(uint64_t ns);
uint64_t spd_get_wait_timeout_ns(void);

/* Exercises the bounded-wait path on the GPU: one CTA waits on a shared-memory barrier
 * phase that nothing completes, gives up after timeout_ns (0 < timeout_ns <= 2 s) and
 * ORs SPD_DEVERR_TIMEOUT into *error_word.  Issues no copy; faults and hangs nothing.
 * For failure-detection tests; no counterpart in the reference. */
int spd_selftest_wait_timeout(int32_t* error_word, uint64_t timeout_ns, void* stream);

/* Copies the device error word of a workspace (or any int32 error word) to *host_word.
 * Synchronises `stream`. Not for use during graph capture. */
int spd_read_error_word(const void* error_word, int32_t* host_word, void* stream);

/* (1) Paged single-query decoder self-attention (+ fused op 3).
 *   q        [B][H][D]            query of the new token (unscaled)
 *   k_pool   [num_blocks][block_size][H][D], v_pool likewise (one decoder layer)
 *   block_tables [B][max_blocks]  int32 physical block ids
 *   context_lens [B]              int32 tokens to attend to, INCLUDING the new token;
 *                                 <= 0 writes zeros to out[b] (the reference kernel skips
 *                                 such rows, leaving its zero-initialised output)
 *   out      [B][H][D]            softmax(q·Kᵀ·scale)·V over positions [0, ctx)
 *   k_new/v_new [B][H][D] or NULL when non-NULL, the new token's K/V is first written
 *                                 to position ctx-1 of its block (op 3 fused) and the
 *                                 attention sees it.
 * Arithmetic: fp32 accumulation, output rounded to `dtype`.
 * Supported: dtype F32/F16/BF16; D in {16,32,64,128}; block_size in {8,16,32};
 * H <= 32; B <= 4096. */
int spd_paged_decode_attn(const void* q, void* k_pool, void* v_pool,
                          const int32_t* block_tables, const int32_t* context_lens,
                          void* out, int B, int H, int D, int block_size, int max_blocks,
                          int num_blocks, float scale, int dtype,
                          const void* k_new, const void* v_new,
                          void* workspace, size_t workspace_bytes, void* stream);

/* (2) Single-query cross-attention over contiguous encoder K/V.
 *   q   [B][H][D];  out [B][H][D]
 *   k,v element (b,h,t,d) at  k + b*kv_batch_stride + h*kv_head_stride + t*D + d
 *       (elements).  The graph-slot layout [S][L][2][H][T_max][D] for layer l is
 *       k = base + l*2*H*T_max*D, v = k + H*T_max*D, kv_batch_stride = L*2*H*T_max*D,
 *       kv_head_stride = T_max*D.
 *   valid_lens [B] int32 positions attended per request (clamped to T_max; <= 0 -> zeros).
 * Supported: dtype F32/F16/BF16; D in {16,32,64,128}; B*H <= 65536. */
int spd_cross_attn(const void* q, const void* k, const void* v, const int32_t* valid_lens,
                   void* out, int B, int H, int D, int T_max, int64_t kv_batch_stride,
                   int64_t kv_head_stride, float scale, int dtype, void* workspace,
                   size_t workspace_bytes, void* stream);

/* (3) Write T tokens of K/V per sequence into their paged blocks (bit-exact copy).
 *   src element (b,h,t,d) at k_src + b*src_stride_b + h*src_stride_h + t*src_stride_t + d
 *   positions [B] int32: first position to write for sequence b (< 0: sequence skipped)
 *   Destination row of (b, t): block_tables[b][(pos+t)/block_size], offset (pos+t)%block_size.
 *   v_src / v_pool may be NULL to write K only.
 *   error_word: optional int32 device word that receives SPD_DEVERR_* flags. */
int spd_kv_append(const void* k_src, const void* v_src, int64_t src_stride_b,
                  int64_t src_stride_h, int64_t src_stride_t, void* k_pool, void* v_pool,
                  const int32_t* block_tables, const int32_t* positions, int B, int T, int H,
                  int D, int block_size, int max_blocks, int num_blocks, int dtype,
                  int32_t* error_word, void* stream);

/* (5) Gather paged blocks into a contiguous head-major tensor (bit-exact copy).
 *   out element (b,h,t,d) at out + b*out_batch_stride + (h*T_out + t)*D + d
 *   = pool[block_tables[b][t/block_size]][t%block_size][h][d]   for t < seq_lens[b]
 *   = 0 for seq_lens[b] <= t < T_out when zero_pad != 0 (untouched otherwise). */
int spd_block_gather(const void* pool, const int32_t* block_tables, const int32_t* seq_lens,
                     void* out, int B, int H, int D, int block_size, int max_blocks,
                     int num_blocks, int T_out, int64_t out_batch_stride, int zero_pad,
                     int dtype, int32_t* error_word, void* stream);

/* (4) Cross-KV projection at encoder handoff: one tcgen05 GEMM for all decoder layers.
 *   enc_out [B][T][d_model]          row-major encoder output (dtype F16 or BF16)
 *   w_kv    [L*2*H*D][d_model]       the k_proj and v_proj weights of every decoder layer
 *                                    stacked in (layer, k|v, head, dim) row order
 *   b_kv    [L*2*H*D] or NULL        bias in the same order (zeros where a projection has
 *                                    none: Whisper's k_proj has no bias, v_proj has one)
 *   out     element (b, l, kv, h, t, d) is written at
 *             out + s*out_slot_stride + (((l*2 + kv)*H + h)*T_out + t)*D + d,
 *           s = slot_ids ? slot_ids[b] : b   — the graph-slot layout [S][L][2][H][T_out][D]
 *   error_word: optional int32 device word receiving SPD_DEVERR_TIMEOUT.
 * fp32 accumulation; output rounded to dtype.  Requires d_model % 64 == 0, D % 8 == 0,
 * T <= T_out, 16-byte aligned pointers and slot stride. */
int spd_cross_kv_project(const void* enc_out, const void* w_kv, const void* b_kv, void* out,
                         const int32_t* slot_ids, int B, int T, int d_model, int L, int H,
                         int D, int T_out, int64_t out_slot_stride, int dtype,
                         int32_t* error_word, void* stream);

/* Residual add fused with the LayerNorm that follows it (decoder-layer glue around the
 * kernels above), one warp per row of `cols` elements (cols * element size a multiple
 * of 16 bytes, cols <= 2048):
 *   x_out[r] = round(x[r] + delta[r])                          (delta NULL: x_out unused)
 *   y[r]     = round((x_out[r] - mean) / sqrt(var + eps) * gamma + beta)
 * mean and var (biased) in fp32 over the rounded x_out; x_out may alias x.  Row r of y
 * starts at y + r * y_ld (0: y_ld = cols; y_ld * element size a multiple of 16 bytes),
 * so y can be the leading columns of a wider buffer. */
int spd_add_layernorm(const void* x, const void* delta, const void* gamma, const void* beta,
                      void* x_out, void* y, int rows, int cols, int64_t y_ld, float eps, int dtype,
                      void* stream);

/* Greedy token pick: out[r] = the first c < cols maximising x[r*ld + c], where a column
 * with skip_mask[c] != 0 (uint8 [cols], or NULL) scores -inf and a NaN beats any number;
 * the same index as torch.argmax(x[:, :cols].masked_fill(skip_mask, -inf), dim=-1).
 * out is int64 [rows]; ld >= cols (elements between rows). */
int spd_argmax_rows(const void* x, int rows, int cols, int64_t ld, const void* skip_mask, int64_t* out,
                    int dtype, void* stream);

/* Small-batch Linear layer (the decode step's projections, MLP and head) on the tensor
 * cores (tcgen05, weights streamed by TMA, K split over a thread-block cluster when N is
 * small):
 *   y(m, n) = act( sum_k x[m*K + k] * w[n*K + k] + bias[n] )   m < M, n < N
 * x [M][K] and w [N][K] row-major (w is an nn.Linear weight), bias [N] or NULL,
 * activation SPD_ACT_NONE or SPD_ACT_GELU (the erf form, as torch's default GELU).
 * Output column n is written to plane n / y_group_cols, planes y_group_stride elements
 * apart, each [M][y_group_cols] (y_group_cols = N: a plain [M][N] output; a packed q|k|v
 * weight with y_group_cols = H*D writes q, k and v as three [M][H*D] tensors).
 * fp32 accumulation, one rounding to dtype.  Requires dtype F16 or BF16, 1 <= M <= 64,
 * K a multiple of 64, N a multiple of y_group_cols, x and w 16-byte aligned.
 * error_word: optional int32 device word receiving SPD_DEVERR_TIMEOUT. */
#define SPD_ACT_NONE 0
#define SPD_ACT_GELU 1
int spd_linear(const void* x, const void* w, const void* bias, void* y, int M, int N, int K,
               int64_t y_group_cols, int64_t y_group_stride, int activation, int dtype,
               int32_t* error_word, void* stream);

/* Allocation-free variant of spd_paged_decode_attn, for callers that cannot allocate
 * GPU memory or own a workspace: code running where cudaMalloc is unavailable or
 * forbidden (inside an allocator callback, a plugin host that hands out only the
 * tensors of the call, a process whose memory budget is fixed up front).  It has no
 * counterpart in the reference, which always allocates through PyTorch.
 *   Same arguments and results as spd_paged_decode_attn, minus the workspace; the
 *   split-KV scratch lives in a 4 MiB array inside the library that every GPU using this
 *   entry point keeps until the process exits (SPD_NOALLOC_SCRATCH_BYTES).  Calls whose
 *   spd_paged_decode_attn_workspace_size(B, H, D, max_blocks, device) exceeds it are
 *   rejected with SPD_ERR_WORKSPACE (e.g. B=64, H=12, D=64, 28 blocks per table needs
 *   about 3.0 MiB); arguments are checked before the scratch is touched.
 *   error_word: optional int32 device word; this call's SPD_DEVERR_* flags are OR-ed into
 *   it (flags already there are kept).
 *   The first call on each device looks up the array's device address; make that first
 *   call before capturing any stream.  The address is cached for the process: calls after
 *   a cudaDeviceReset are not supported.  Every call clears the scratch counters it needs,
 *   and all calls share one array: calls that overlap on the GPU (different streams, or
 *   several host threads) race and give wrong results. */
#define SPD_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)
int spd_paged_decode_attn_noalloc(const void* q, void* k_pool, void* v_pool,
                                  const int32_t* block_tables, const int32_t* context_lens,
                                  void* out, int B, int H, int D, int block_size,
                                  int max_blocks, int num_blocks, float scale, int dtype,
                                  const void* k_new, const void* v_new, int32_t* error_word,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPD_B200_H */
