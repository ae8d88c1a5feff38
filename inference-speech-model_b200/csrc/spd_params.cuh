// spd_params.cuh — kernel parameter blocks shared by the kernels and the ABI layer.
// Passed to kernels by value (they live in the constant parameter bank).
#pragma once

#include "spd_common.cuh"

namespace spd {

struct PagedParams {
  const void* q;
  void* k_pool;
  void* v_pool;
  const int* block_tables;
  const int* context_lens;
  void* out;
  const void* k_new;
  const void* v_new;
  int B, H, max_blocks, num_blocks;
  float scale_log2;  // scale * log2(e)
  int* err;          // workspace error word
  int* work;         // [0] next item to take, [1] CTAs done taking (both left at zero)
  int* counters;     // [B * H] ints kept in the workspace layout; the current kernels leave them unused
  float* partials;   // [B * ceil(max_blocks / kItemUnits) * H * (D + 8)]
  int stages;
  int table_in_smem;  // the whole block table is bulk-copied into shared memory
  unsigned long long wait_ns;  // bound on each wait that makes progress
};

struct CrossParams {
  const void* q;
  const void* k;
  const void* v;
  const int* valid_lens;
  void* out;
  int B, H, T_max;
  long long kv_batch_stride, kv_head_stride;  // elements
  float scale_log2;
  int* err;
  int* work;        // [0] next item to take, [1] CTAs done taking (both left at zero)
  float* partials;  // [B*H*kCrossMaxItems * (D + 2)]: one row per item
  int stages;
  int item_units;   // units (of the kernel's row chunk) per work item
  unsigned long long wait_ns;  // bound on each wait that makes progress
};

struct AppendParams {
  const unsigned char* k_src;
  const unsigned char* v_src;
  long long sb, sh, st;  // source strides in bytes
  unsigned char* k_pool;
  unsigned char* v_pool;
  const int* block_tables;
  const int* positions;
  int B, T, H, row_bytes, block_size, max_blocks, num_blocks;
  int* err;
};

struct AddLnParams {  // residual add + LayerNorm (decoder_layer_ops.cu)
  const void* x;
  const void* delta;  // or null: y = LayerNorm(x), x_out not written
  const void* gamma;
  const void* beta;
  void* x_out;
  void* y;
  int rows, cols;
  long long y_ld;  // elements between rows of y
  float eps;
};

struct ArgmaxParams {  // greedy token pick over rows (decoder_layer_ops.cu)
  const void* x;
  const void* skip;  // uint8 [cols] or null: columns scored as -inf
  long long* out;    // int64 [rows]
  int rows, cols;
  long long ld;      // elements between rows
  int vec;           // rows start 16-byte aligned: 16-byte loads
};

struct GatherParams {
  const unsigned char* pool;
  const int* block_tables;
  const int* seq_lens;
  unsigned char* out;
  int B, H, row_bytes, block_size, max_blocks, num_blocks, T_out, zero_pad;
  long long out_batch_stride;  // bytes
  int* err;
};

}  // namespace spd
