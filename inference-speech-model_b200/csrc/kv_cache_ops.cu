// kv_cache_ops.cu — op (3) paged K/V write and op (5) block gather.  Both are pure,
// bit-exact copies between the paged pool layout [num_blocks][block_size][H][D] and
// head-major token rows; they move 16-byte vectors with one thread per vector and
// validate every block id / position on the device (bad entries are skipped and
// recorded in the error word instead of faulting).
//
// op (3) replaces the per-request Python loop that writes the new token's K/V into
// key_pool[l][blk, off] (speech_serving/phase_aware_scheduler.py:1004-1010), the prompt
// block writes (:678-690), the graph path's scatter_ at the clamped position
// (speech_serving/models.py:449-454, speech_serving/graph_decode_buffers.py:56-59) and
// EncoderBlockManager.store_encoder_kv (speech_serving/encoder_block_manager.py:177-192).
//
// op (5) replaces pool[table].view(-1, H, D)[:T].permute(1, 0, 2) with the zero-padded
// batched form (speech_serving/phase_aware_scheduler.py:613-624, :859-882, :926-962;
// speech_serving/encoder_attention.py:50-63).
#include "spd_params.cuh"

namespace spd {

// One thread per 16-byte (VB-byte) vector of one (b, t, h) row; K and V together.
template <int VB>
__global__ void kv_append_kernel(const AppendParams p) {
  const int vpr = p.row_bytes / VB;  // vectors per row
  const long long total = (long long)p.B * p.T * p.H * vpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = (int)(i % vpr);
    long long rest = i / vpr;
    const int h = (int)(rest % p.H);
    rest /= p.H;
    const int t = (int)(rest % p.T);
    const int b = (int)(rest / p.T);
    const int p0 = p.positions[b];
    if (p0 < 0) continue;
    const long long pos = (long long)p0 + t;
    const long long blk = pos / p.block_size;
    if (blk >= p.max_blocks) {
      if (v == 0) set_error(p.err, SPD_DEVERR_LENGTH);
      continue;
    }
    const int phys = p.block_tables[(long long)b * p.max_blocks + blk];
    if (phys < 0 || phys >= p.num_blocks) {
      if (v == 0) set_error(p.err, SPD_DEVERR_BLOCK_ID);
      continue;
    }
    const long long dst =
        (((long long)phys * p.block_size + pos % p.block_size) * p.H + h) * p.row_bytes + (long long)v * VB;
    const long long src = b * p.sb + h * p.sh + t * p.st + (long long)v * VB;
    if constexpr (VB == 16) {
      *reinterpret_cast<uint4*>(p.k_pool + dst) = *reinterpret_cast<const uint4*>(p.k_src + src);
      if (p.v_pool) *reinterpret_cast<uint4*>(p.v_pool + dst) = *reinterpret_cast<const uint4*>(p.v_src + src);
    } else if constexpr (VB == 4) {
      *reinterpret_cast<uint32_t*>(p.k_pool + dst) = *reinterpret_cast<const uint32_t*>(p.k_src + src);
      if (p.v_pool)
        *reinterpret_cast<uint32_t*>(p.v_pool + dst) = *reinterpret_cast<const uint32_t*>(p.v_src + src);
    } else {
      *reinterpret_cast<uint16_t*>(p.k_pool + dst) = *reinterpret_cast<const uint16_t*>(p.k_src + src);
      if (p.v_pool)
        *reinterpret_cast<uint16_t*>(p.v_pool + dst) = *reinterpret_cast<const uint16_t*>(p.v_src + src);
    }
  }
}

// One thread per 16-byte vector of one output row (b, h, t); consecutive threads walk
// the D dimension then t, so each warp writes contiguous output.
__global__ void block_gather_kernel(const GatherParams p) {
  const int vpr = p.row_bytes / 16;
  const long long total = (long long)p.B * p.H * p.T_out * vpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = (int)(i % vpr);
    long long rest = i / vpr;
    const int t = (int)(rest % p.T_out);
    rest /= p.T_out;
    const int h = (int)(rest % p.H);
    const int b = (int)(rest / p.H);
    unsigned char* dst = p.out + b * p.out_batch_stride + ((long long)h * p.T_out + t) * p.row_bytes + v * 16;
    const int len = p.seq_lens[b];
    if (t >= len) {
      if (p.zero_pad) *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int blk = t / p.block_size;
    if (blk >= p.max_blocks) {
      if (v == 0) set_error(p.err, SPD_DEVERR_LENGTH);
      continue;
    }
    const int phys = p.block_tables[(long long)b * p.max_blocks + blk];
    if (phys < 0 || phys >= p.num_blocks) {
      if (v == 0) set_error(p.err, SPD_DEVERR_BLOCK_ID);
      continue;
    }
    const unsigned char* src =
        p.pool + (((long long)phys * p.block_size + t % p.block_size) * p.H + h) * p.row_bytes + v * 16;
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  }
}

static int grid_for(long long total, int threads, int sms) {
  long long g = (total + threads - 1) / threads;
  const long long cap = (long long)sms * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

int kv_append_launch(const AppendParams& p, int sms, cudaStream_t st) {
  const bool a16 = (p.row_bytes % 16 == 0) && (p.sb % 16 == 0) && (p.sh % 16 == 0) && (p.st % 16 == 0) &&
                   ((uintptr_t)p.k_src % 16 == 0) && (!p.v_src || (uintptr_t)p.v_src % 16 == 0);
  const bool a4 = (p.row_bytes % 4 == 0) && (p.sb % 4 == 0) && (p.sh % 4 == 0) && (p.st % 4 == 0) &&
                  ((uintptr_t)p.k_src % 4 == 0) && (!p.v_src || (uintptr_t)p.v_src % 4 == 0);
  const int threads = 256;
  const int vb = a16 ? 16 : (a4 ? 4 : 2);
  const long long total = (long long)p.B * p.T * p.H * (p.row_bytes / vb);
  if (total == 0) return SPD_OK;
  const int grid = grid_for(total, threads, sms);
  if (a16) kv_append_kernel<16><<<grid, threads, 0, st>>>(p);
  else if (a4) kv_append_kernel<4><<<grid, threads, 0, st>>>(p);
  else kv_append_kernel<2><<<grid, threads, 0, st>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

int block_gather_launch(const GatherParams& p, int sms, cudaStream_t st) {
  const int threads = 256;
  const long long total = (long long)p.B * p.H * p.T_out * (p.row_bytes / 16);
  if (total == 0) return SPD_OK;
  block_gather_kernel<<<grid_for(total, threads, sms), threads, 0, st>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

}  // namespace spd
