// linear_small_m.cu — the decode step's Linear layers for small batches (M <= 64 rows) as
// a weight-streaming tcgen05 GEMM:
//   Y[m, n] = act( sum_k X[m, k] * W[n, k] + bias[n] ),   X [M][K], W [N][K] (nn.Linear)
//
// Replaces the per-layer projections of the reference's decode step
// (speech_serving/models.py:127-129 q/k/v, :159 self out, :178-180 cross q, :202 cross
// out, :205-207 MLP; transformers' WhisperDecoderLayer likewise) and the output head.
// At M <= 64 these are bounded by streaming W from HBM, not by the tensor cores.
//
// sm_100a design:
// * A CTA owns 128 output features (the MMA's M) and a K range; X (<= 64 rows, padded by
//   the TMA's zero fill) is the MMA's N = 64.  Warp 0 lane 0 streams 64-wide K slices of
//   W and X with 2-D TMA loads (128-byte swizzle, no multicast) through a 4-stage ring;
//   warp 1 lane 0 issues tcgen05.mma (kind::f16, fp32 accumulation in 64 TMEM columns).
// * Small N leaves most SMs idle, so K is split over a thread-block cluster of ks CTAs
//   (ks in 1..8, chosen so the grid fills the SMs).  Every rank arms its receive barrier
//   and the cluster synchronises once in the prologue, before griddepcontrol.wait (the
//   partial tile and the receive buffer have their own shared memory, past the ring).
//   Once its fp32 partial tile is in shared memory, each rank pushes to rank r the slice
//   of features [r*128/ks, (r+1)*128/ks) with a bulk shared::cluster copy that completes
//   on rank r's mbarrier.  Rank r then sums its features over all ranks from its own
//   shared memory, adds the bias, applies the activation, rounds once and stores.  A
//   cluster barrier at the end keeps every rank alive until the copies it sent have
//   landed.
// * Launched with programmatic dependent launch: before griddepcontrol.wait the CTA only
//   sets up barriers and TMEM and prefetches its W slices into L2 (a hint: the tiles and
//   the bias are read after the wait, so results never depend on what the previous kernel
//   writes).
// * Output columns may be grouped: column n goes to plane n / group_cols (planes
//   group_stride elements apart) as [M][group_cols] — how a packed q|k|v weight writes
//   three separate [M][H*D] tensors.
// * Every mbarrier wait is bounded (SPD_DEVERR_TIMEOUT); a CTA whose wait gave up still
//   takes part in both cluster barriers, so no CTA of its cluster waits forever.
#include <vector>

#include "spd_tc.cuh"
#include "spd_trace.cuh"

// Timeline marks (trace builds only; see spd_trace.cuh), per CTA: 0 entry, 1 set-up done,
// 2 griddepcontrol.wait returned, 3 first stage landed (MMA issuer), 4 accumulator ready,
// 5 partial tiles exchanged (first cluster barrier), 6 outputs stored, 7 exit.
SPD_TRACE_ARRAY
#define LIN_TRACE(point) SPD_TRACE_AT(0, point)

namespace spd {
namespace lin {
using namespace tc;

constexpr int BF = 128;  // output features per CTA (MMA M)
constexpr int BR = 64;   // rows of X per tile (MMA N)
constexpr int STAGES = 4;
constexpr int W_BYTES = BF * BK * 2;  // 16 KB
constexpr int X_BYTES = BR * BK * 2;  // 8 KB
constexpr int PSTRIDE = BR + 4;       // floats per feature row of the partial tile (16-byte aligned rows)
constexpr int RING_BYTES = STAGES * (W_BYTES + X_BYTES);
constexpr int PART_BYTES = BF * PSTRIDE * 4;
// the partial tile and the receive buffer sit after the ring, so peers may push into a
// rank's receive buffer while its MMAs still read the ring
constexpr size_t SMEM_BYTES = 1024 /*alignment slack*/ + RING_BYTES + 2 * PART_BYTES + 256;
constexpr int kThreads = 128;
constexpr int kMaxClusterK = 8;

struct Params {
  const void* bias;  // [N] or null
  void* y;
  int M, N, K;
  long long group_cols, group_stride;  // output column grouping (elements)
  int act;                             // SPD_ACT_*
  int* err;
};

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in cluster rank `rank`'s shared memory.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
  return remote;
}

// Bulk copy of `bytes` from this CTA's shared memory into another cluster CTA's shared
// memory (both addresses 16-byte aligned, bytes a multiple of 16), completing as
// transaction bytes on an mbarrier that lives in the destination CTA.
__device__ __forceinline__ void bulk_copy_s2peer(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(smem_addr(src)), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ float activate(float x, int act) {
  if (act == SPD_ACT_GELU) return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
  return x;
}

template <typename T, int KS>
__global__ void __launch_bounds__(kThreads, 1)
    linear_small_m_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                          const Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_addr = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (base_addr & 1023)) & 1023);  // 1024-aligned for SW128
  unsigned char* w_tiles = smem;
  unsigned char* x_tiles = smem + STAGES * W_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + RING_BYTES + 2 * PART_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* recv_bar = acc_full + 1;  // the peers' slices of this CTA's features have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  // after the ring: this CTA's partial tile [BF][PSTRIDE], then the receive buffer, one
  // [BF / ks][PSTRIDE] slice per cluster rank
  float* part = reinterpret_cast<float*>(smem + RING_BYTES);
  float* recv = part + BF * PSTRIDE;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int ks = KS;
  const int kr = (int)blockIdx.x % ks;  // rank in the cluster = K range
  const int n0 = ((int)blockIdx.x / ks) * BF;
  const int kper = p.K / BK / ks;
  const int kb0 = kr * kper;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  if (tid == 0) LIN_TRACE(0);
  if (warp == 1) tmem_alloc(tmem_slot, BR);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(recv_bar, 1);
    fence_barrier_init();
    for (int i = 0; i < kper; ++i) tma_prefetch_2d(&tm_w, (kb0 + i) * BK, n0);
  }
  // every rank's receive barrier is armed before any peer can push into it: the cluster
  // barrier for that runs here, while the previous kernel in the stream may still run
  constexpr int F = BF / KS;
  constexpr uint32_t kSliceBytes = F * PSTRIDE * 4;
  if (KS > 1 && tid == 0) mbar_arrive_expect_tx(recv_bar, (uint32_t)(KS - 1) * kSliceBytes);
  tc_fence_before();
  __syncthreads();
  if (KS > 1) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) LIN_TRACE(1);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) LIN_TRACE(2);
  // the bias of the feature this thread stores: loaded now, used only in the epilogue
  const int n = n0 + kr * F + tid % F;
  const float bn = (p.bias && n < p.N) ? Elem<T>::to_f(__ldg(reinterpret_cast<const T*>(p.bias) + n)) : 0.f;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ------------------------------------------------------------------
    int i = 0;
    for (; i < kper; ++i) {
      const int s = i % STAGES;
      if (i >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / STAGES) & 1) ^ 1), p.err)) break;
      mbar_arrive_expect_tx(&full[s], W_BYTES + X_BYTES);
      tma_load_2d(w_tiles + s * W_BYTES, &tm_w, (kb0 + i) * BK, n0, &full[s]);
      tma_load_2d(x_tiles + s * X_BYTES, &tm_x, (kb0 + i) * BK, 0, &full[s]);
    }
    if (i < kper)  // a wait gave up: let the copies in flight land before the CTA can exit
      for (int k = i - 1; k >= 0 && k >= i - STAGES; --k)
        (void)mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1), nullptr);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ------------------------------------------------------------------
    constexpr uint32_t idesc = instr_desc_f16(kBf16, BF, BR);
    bool ok = true;
    for (int i = 0; i < kper; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait_bounded(&full[s], (uint32_t)((i / STAGES) & 1), p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (i == 0) LIN_TRACE(3);
      const uint64_t dw = smem_desc_sw128(w_tiles + s * W_BYTES);
      const uint64_t dx = smem_desc_sw128(x_tiles + s * X_BYTES);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) umma_f16(tmem, dw + 2 * k, dx + 2 * k, idesc, (i | k) != 0);
      umma_commit(&empty[s]);
    }
    if (ok) umma_commit(acc_full);
  }
  __syncwarp();

  // ---- accumulator -> this CTA's partial tile in shared memory [feature][row] -----------
  const bool ready = mbar_wait_bounded(acc_full, 0, p.err);
  const bool all_ready = __syncthreads_and(ready ? 1 : 0) != 0;
  tc_fence_after();
  if (tid == 0) LIN_TRACE(4);
  if (all_ready) {
    const int f = warp * 32 + lane;  // TMEM lane = feature row of the tile
#pragma unroll
    for (int c0 = 0; c0 < BR; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(part + f * PSTRIDE + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }
  fence_proxy_async_smem();  // the partial tile is read by bulk copies (async proxy) next
  // ---- exchange: rank r receives every peer's slice of features [r*F, (r+1)*F) ---------
  // Each rank pushes its slices with bulk shared-to-shared copies (the copy engine, not
  // per-thread remote loads) into receive buffers armed in the prologue; the CTA barrier
  // orders this CTA's partial-tile writes before its copies read them.  Every rank sends
  // even when its own accumulator was not ready, so every receive barrier completes.
  __syncthreads();
  if (ks > 1) {
    if (tid < ks && tid != kr) {
      const uint32_t peer = (uint32_t)tid;
      bulk_copy_s2peer(dsmem_addr(recv + kr * F * PSTRIDE, peer), part + tid * F * PSTRIDE, kSliceBytes,
                       dsmem_addr(recv_bar, peer));
    }
  }
  if (tid == 0) LIN_TRACE(5);
  const bool got = ks == 1 || mbar_wait_bounded(recv_bar, 0, p.err);

  // ---- rank kr: its features summed over the cluster, bias, act, store ------------------
  // Thread t owns feature kr*F + t % F and the row quads t / F, t / F + KS, ...: its 16
  // vector loads (own partial and received slices, all local) are issued before any is
  // used; the bias is read once; for a fixed row consecutive threads store consecutive
  // features.
  constexpr int QPT = (BR / 4) / KS;  // row quads per thread
  const int M = p.M;
  const int fl = tid % F, q0 = tid / F;
  const int f = kr * F + fl;
  if (all_ready && got && n < p.N) {
    float4 acc4[QPT][KS];
#pragma unroll
    for (int r = 0; r < KS; ++r) {
      const float* row = r == kr ? part + f * PSTRIDE : recv + (r * F + fl) * PSTRIDE;
#pragma unroll
      for (int j = 0; j < QPT; ++j) acc4[j][r] = *reinterpret_cast<const float4*>(row + (q0 + j * KS) * 4);
    }
    const long long g = n / p.group_cols, c = n % p.group_cols;
    T* yc = reinterpret_cast<T*>(p.y) + g * p.group_stride + c;
#pragma unroll
    for (int j = 0; j < QPT; ++j) {
      float4 sum = acc4[j][0];
#pragma unroll
      for (int r = 1; r < KS; ++r) {
        sum.x += acc4[j][r].x;
        sum.y += acc4[j][r].y;
        sum.z += acc4[j][r].z;
        sum.w += acc4[j][r].w;
      }
      const float o[4] = {sum.x, sum.y, sum.z, sum.w};
      const int m0 = (q0 + j * KS) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (m0 + i < M) yc[(long long)(m0 + i) * p.group_cols] = Elem<T>::from_f(activate(o[i] + bn, p.act));
    }
  }
  if (tid == 0) LIN_TRACE(6);
  // the copies this CTA sent have landed once every rank has passed its receive wait
  if (ks > 1) cluster_sync();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, BR);
  if (tid == 0) LIN_TRACE(7);
}

}  // namespace lin

int linear_small_m_launch(const void* x, const void* w, const void* bias, void* y, int M, int N, int K,
                          long long group_cols, long long group_stride, int act, int dtype, int* err, int sms,
                          cudaStream_t st) {
  using namespace lin;
  const bool bf16 = dtype == SPD_BF16;
  const int tiles = (N + BF - 1) / BF;
  const int nk = K / BK;
  // split K over a cluster until the grid covers the SMs (K slices must divide evenly)
  int ks = 1;
  while (ks < kMaxClusterK && tiles * ks * 2 <= sms && nk % (ks * 2) == 0) ks *= 2;
  CUtensorMap tw, tx;
  if (!make_map(&tw, w, K, N, BF, bf16) || !make_map(&tx, x, K, M, BR, bf16)) return SPD_ERR_CUDA;
  Params p{};
  p.bias = bias; p.y = y; p.M = M; p.N = N; p.K = K;
  p.group_cols = group_cols; p.group_stride = group_stride; p.act = act; p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * ks));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  auto launch = [&](auto kfn) -> int {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
      return SPD_ERR_CUDA;
    return cudaLaunchKernelEx(&cfg, kfn, tw, tx, p) == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
  };
  auto by_ks = [&](auto tag) -> int {
    using T = decltype(tag);
    switch (ks) {
      case 1: return launch(linear_small_m_kernel<T, 1>);
      case 2: return launch(linear_small_m_kernel<T, 2>);
      case 4: return launch(linear_small_m_kernel<T, 4>);
      default: return launch(linear_small_m_kernel<T, 8>);
    }
  };
  return bf16 ? by_ks(__nv_bfloat16{}) : by_ks(__half{});
}

}  // namespace spd

#ifdef SPD_TRACE_BUILD
// Trace builds only: copies the last launch's marks ([kernel][CTA][point], %globaltimer
// values, 0 where a mark was not reached) into `host` and clears them (synchronous).
extern "C" int spd_trace_fetch_linear(unsigned long long* host, size_t count) {
  const size_t n = (size_t)spd::kTraceKernels * spd::kTraceCtas * spd::kTracePoints;
  if (!host || count < n) return SPD_ERR_INVALID_ARG;
  if (cudaMemcpyFromSymbol(host, spd::g_trace, n * sizeof(unsigned long long)) != cudaSuccess) return SPD_ERR_CUDA;
  std::vector<unsigned long long> zero(n, 0ull);
  return cudaMemcpyToSymbol(spd::g_trace, zero.data(), n * sizeof(unsigned long long)) == cudaSuccess ? SPD_OK
                                                                                                     : SPD_ERR_CUDA;
}
#endif
