// cross_kv_project.cu — op (4): the cross-KV projection at encoder handoff as one
// tcgen05 GEMM over every decoder layer.
//
// Reference: speech_serving/models.py:554-561 runs, per decoder layer,
//   k = encoder_attn.k_proj(enc_out)   (no bias)      -> view [B,T,H,D] -> transpose(1,2)
//   v = encoder_attn.v_proj(enc_out)   (+ bias)       -> view [B,T,H,D] -> transpose(1,2)
// i.e. 2*L GEMMs [B*T, d] x [d, H*D] plus 2*L transpose copies.  Here the k_proj/v_proj
// weights of all layers are stacked into W [L*2*H*D, d] and ONE GEMM
//   C[m, n] = sum_k A[m, k] * W[n, k] + bias[n],   A = enc_out viewed [B*T, d]
// is computed, with the epilogue writing C straight into the graph-slot layout
// [S][L][2][H][T_out][D] (no transpose copies).
//
// sm_100a design: a persistent grid (one CTA per SM) walks the 128x256 output tiles.
// Warp 0 lane 0 issues 2-D TMA loads (128-byte swizzle, no multicast) of the A and W
// tiles for each 64-wide K slice into a 4-stage shared-memory ring (full/empty
// mbarriers); warp 1 lane 0 issues tcgen05.mma (kind::f16, M=128, N=256, K=16) into one
// of two 256-column fp32 TMEM accumulators, frees each stage with tcgen05.commit and
// signals a finished tile with a commit on that accumulator's barrier; warps 2..9 are
// the epilogue, one accumulator row (TMEM lane) and half the columns per thread: tcgen05.ld, the bias in
// fp32, rounding, and 16-byte stores of one head's row into the slot layout, after which
// the accumulator is handed back.  So tile i's epilogue overlaps tile i+1's MMAs.  All
// waits are bounded (SPD_DEVERR_TIMEOUT on expiry).
//
// From d_model 1024 up a second form runs the same GEMM on 2-CTA clusters with
// tcgen05.mma.cta_group::2 over 256 x 256 tiles (cross_kv_project_pair_kernel below):
// each CTA stages half of A's and half of W's rows, so a stage is 32 KB instead of 48 KB
// for the same MMA work per SM.
#include "spd_tc.cuh"

namespace spd {

namespace proj {
using namespace tc;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 256;
constexpr size_t SMEM_BYTES = 1024 /*alignment slack*/ + (size_t)STAGES * (A_BYTES + B_BYTES) + 256;

struct Params {
  const void* bias;      // [N] or null
  void* out;
  const int* slot_ids;   // [B] or null
  int M, N, K, T, H, D, T_out;
  long long out_slot_stride;  // elements
  int* err;
};

// Instruction descriptor: M = 128, N = BN.
__host__ __device__ constexpr uint32_t instr_desc(bool bf16) { return instr_desc_f16(bf16, BM, BN); }

// Epilogue of one accumulator row: columns [n, n + C) of output row `out` (already offset
// to the row's slot and position): + bias in fp32, one rounding, 16-byte stores of eight
// consecutive head dimensions into the slot layout [L][2][H][T_out][D].
template <typename T, int C>
__device__ __forceinline__ void store_row_chunk(const float* v, int n_first, int N, int HD, int H, int D,
                                                long long plane, const T* bias, T* out) {
#pragma unroll
  for (int g = 0; g < C; g += 8) {
    const int n = n_first + g;
    if (n >= N) break;
    const int lkv = n / HD, rem = n % HD;
    const int h = rem / D, d = rem % D;
    alignas(16) T o[8];
    if (bias) {
      alignas(16) T bb[8];
      *reinterpret_cast<uint4*>(bb) = __ldg(reinterpret_cast<const uint4*>(bias + n));
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = Elem<T>::from_f(v[g + i] + Elem<T>::to_f(bb[i]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = Elem<T>::from_f(v[g + i]);
    }
    *reinterpret_cast<uint4*>(out + ((long long)lkv * H + h) * plane + d) = *reinterpret_cast<uint4*>(o);
  }
}

// Persistent, warp-specialised: CTA c computes tiles c, c + G, c + 2G, ... (G CTAs).
//   warp 0        TMA producer: A and W K-slices into the STAGES-deep shared ring
//   warp 1        MMA issuer: each tile into one of two TMEM accumulators (2 x 256 columns)
//   warps 2..     epilogue: TMEM -> registers -> bias -> slot layout; warp w reads TMEM
//                 lanes 32*(w%4).., so each group of four warps covers the 128
//                 accumulator rows, and the groups split the columns
// The epilogue of tile i runs while the MMAs of tile i+1 fill the other accumulator.
#ifndef SPD_PROJ_EPI_WARPS
#define SPD_PROJ_EPI_WARPS 8
#endif
// Epilogue warps: 4 or 8 (or 16).  Warp w may only read TMEM lanes 32*(w%4).., so with 8
// the two warps of a lane quarter split the accumulator's columns.  Eight drain a tile
// fast enough that the MMAs no longer wait for the accumulator (Whisper-small handoff
// 68 -> 52.5 us, large-v3 341 -> 277.5 us per request, against four).
constexpr int kEpiWarps = SPD_PROJ_EPI_WARPS;
constexpr int kProjThreads = 64 + 32 * kEpiWarps;
constexpr int kAccBufs = 2;
#ifndef SPD_PROJ_PAIRS
#define SPD_PROJ_PAIRS 1
#endif
constexpr bool kProjPairs = SPD_PROJ_PAIRS != 0;  // use the CTA-pair form when it launches
#ifndef SPD_PROJ_PAIR_MIN_K
#define SPD_PROJ_PAIR_MIN_K 1024
#endif
constexpr int kPairMinK = SPD_PROJ_PAIR_MIN_K;     // ... and d_model is at least this

template <typename T>
__global__ void __launch_bounds__(kProjThreads, 1)
    cross_kv_project_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                            const Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_addr = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (base_addr & 1023)) & 1023);  // 1024-aligned for SW128
  unsigned char* a_tiles = smem;
  unsigned char* b_tiles = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_tiles + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;     // [kAccBufs]: MMAs of a tile done
  uint64_t* acc_empty = acc_full + kAccBufs;  // [kAccBufs]: epilogue has read the accumulator
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kAccBufs);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = p.K / BK;
  const int tiles_n = (p.N + BN - 1) / BN, tiles_m = (p.M + BM - 1) / BM;
  const int n_tiles = tiles_n * tiles_m;
  constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;

  if (warp == 1) tmem_alloc(tmem_slot, kAccBufs * TMEM_COLS);
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer --------------------------------------------------------------
    if (lane == 0) {
      long long it = 0;  // K-slices issued, over all tiles
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          if (it >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((it / STAGES) & 1) ^ 1), p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
          tma_load_2d(a_tiles + s * A_BYTES, &tm_a, kb * BK, m0, &full[s]);
          tma_load_2d(b_tiles + s * B_BYTES, &tm_b, kb * BK, n0, &full[s]);
        }
      }
      if (!ok)  // let the copies in flight land before the CTA can exit
        for (long long k = it - 1; k >= 0 && k >= it - STAGES; --k)
          (void)mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1), nullptr);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(kBf16);
      long long it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local % kAccBufs;
        const int use = local / kAccBufs;
        if (use > 0 && !mbar_wait_bounded(&acc_empty[buf], (uint32_t)((use - 1) & 1), p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(buf * TMEM_COLS);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          if (!mbar_wait_bounded(&full[s], (uint32_t)((it / STAGES) & 1), p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(a_tiles + s * A_BYTES);
          const uint64_t db = smem_desc_sw128(b_tiles + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // each K=16 step advances 32 bytes inside the 128-byte swizzle row
            umma_f16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ---- epilogue: thread = accumulator row (TMEM lane 32*(warp%4) + lane) ---------------
    const int q = warp & 3;
    constexpr int kCols = BN * 4 / kEpiWarps;  // accumulator columns per epilogue warp
    const int c_begin = ((warp - 2) / 4) * kCols;
    const T* bias = reinterpret_cast<const T*>(p.bias);
    const int HD = p.H * p.D;
    const long long plane = (long long)p.T_out * p.D;  // one (layer, k|v, head) plane
    int local = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++local) {
      const int buf = local % kAccBufs;
      const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
      const bool ready = mbar_wait_bounded(&acc_full[buf], (uint32_t)((local / kAccBufs) & 1), p.err);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int m = m0 + q * 32 + lane;
      const bool row_ok = m < p.M;
      const int b = row_ok ? m / p.T : 0;
      const int t = row_ok ? m % p.T : 0;
      const long long slot = row_ok ? (p.slot_ids ? p.slot_ids[b] : b) : 0;
      T* out = reinterpret_cast<T*>(p.out) + slot * p.out_slot_stride + (long long)t * p.D;
#pragma unroll 1
      for (int c0 = c_begin; c0 < c_begin + kCols; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TMEM_COLS + c0), v);  // all lanes
        if (!row_ok) continue;
#pragma unroll
        for (int g = 0; g < 16; g += 8) {
          const int n = n0 + c0 + g;
          if (n >= p.N) break;
          const int lkv = n / HD, rem = n % HD;
          const int h = rem / p.D, d = rem % p.D;
          alignas(16) T o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float x = v[g + i];
            if (bias) x += Elem<T>::to_f(bias[n + i]);
            o[i] = Elem<T>::from_f(x);
          }
          *reinterpret_cast<uint4*>(out + ((long long)lkv * p.H + h) * plane + d) = *reinterpret_cast<uint4*>(o);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kAccBufs * TMEM_COLS);
}


// ---- the CTA-pair form -------------------------------------------------------------
// A 2-CTA cluster computes 256 x 256 output tiles with tcgen05.mma.cta_group::2: rank r
// stages rows [128r, 128r + 128) of the A tile and rows [128r, 128r + 128) of the 256-row
// W tile (16 KB + 16 KB per 64-wide K slice instead of 16 KB + 32 KB for a one-CTA
// 128 x 256 tile), rank 0 issues the MMAs (M = 256, N = 256), and each CTA's TMEM receives
// its 128 rows of the tile across all 256 columns.  So each CTA moves a third fewer bytes
// from L2 per FLOP, and still double-buffers its accumulator (2 x 256 TMEM columns).
//   warp 0        TMA producer of this CTA's halves; both CTAs' loads complete on rank 0's
//                 full barrier (rank 0 arms it for both)
//   warp 1        rank 0: MMA issuer; each stage is released to both producers and each
//                 finished tile to both epilogues by one tcgen05.commit per CTA
//   warps 2..     epilogue of this CTA's 128 rows; every epilogue warp of each CTA
//                 arrives on rank 0's accumulator-empty barrier
// Every wait is bounded.  On an error both CTAs still pass both cluster barriers, and
// rank 0 waits (bounded) for the stages either producer issued before the CTAs exit, so
// no copy lands in the shared memory of a CTA that has left.
#ifndef SPD_PROJ_PAIR_STAGES
#define SPD_PROJ_PAIR_STAGES 6
#endif
#ifndef SPD_PROJ_PAIR_MMAJOR
#define SPD_PROJ_PAIR_MMAJOR 1
#endif
constexpr int P_STAGES = SPD_PROJ_PAIR_STAGES;
constexpr int P_ROWS = 128;                 // A rows and W rows per CTA per tile
constexpr int P_A_BYTES = P_ROWS * BK * 2;  // 16 KB
constexpr int P_B_BYTES = P_ROWS * BK * 2;  // 16 KB
constexpr int P_TILE_M = 2 * P_ROWS, P_TILE_N = 2 * P_ROWS;
// tile -> output origin: M-major (consecutive pairs share a W tile; measured faster than
// N-major at large-v3: 357 against 387 us) or N-major (consecutive pairs share an A row block)
__device__ __forceinline__ int pair_n0(int tile, int tiles_n, int tiles_m) {
  return (SPD_PROJ_PAIR_MMAJOR ? tile / tiles_m : tile % tiles_n) * P_TILE_N;
}
__device__ __forceinline__ int pair_m0(int tile, int tiles_n, int tiles_m) {
  return (SPD_PROJ_PAIR_MMAJOR ? tile % tiles_m : tile / tiles_n) * P_TILE_M;
}
constexpr size_t P_SMEM_BYTES = 1024 + (size_t)P_STAGES * (P_A_BYTES + P_B_BYTES) + 256;

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kProjThreads, 1)
    cross_kv_project_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                                 const Params p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_addr = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + ((1024 - (base_addr & 1023)) & 1023);  // same offsets in both CTAs
  unsigned char* a_tiles = smem;
  unsigned char* b_tiles = smem + P_STAGES * P_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_tiles + P_STAGES * P_B_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* acc_full = empty + P_STAGES;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kAccBufs);
  long long* issued_slot = reinterpret_cast<long long*>(tmem_slot + 2);  // 8-byte aligned

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int nk = p.K / BK;
  const int tiles_n = (p.N + P_TILE_N - 1) / P_TILE_N, tiles_m = (p.M + P_TILE_M - 1) / P_TILE_M;
  const int n_tiles = tiles_n * tiles_m;
  const int pair = (int)blockIdx.x / 2, pairs = (int)gridDim.x / 2;
  constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;

  if (warp == 1) tmem_alloc_pair(tmem_slot, kAccBufs * TMEM_COLS);
  if (tid == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);  // rank 0's: the epilogue warps of both CTAs
    }
    *issued_slot = 0;
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  cluster_barrier();  // rank 0's barriers are initialised before any copy signals them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer (both ranks) ---------------------------------------------------
    if (lane == 0) {
      long long it = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += pairs) {
        const int n0 = pair_n0(tile, tiles_n, tiles_m), m0 = pair_m0(tile, tiles_n, tiles_m);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % P_STAGES);
          if (it >= P_STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((it / P_STAGES) & 1) ^ 1), p.err)) {
            ok = false;
            break;
          }
          const uint32_t bar0 = peer_addr(&full[s], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (P_A_BYTES + P_B_BYTES));
          tma_load_2d_pair(a_tiles + s * P_A_BYTES, &tm_a, kb * BK, m0 + (int)rank * P_ROWS, bar0);
          tma_load_2d_pair(b_tiles + s * P_B_BYTES, &tm_b, kb * BK, n0 + (int)rank * P_ROWS, bar0);
        }
      }
      *issued_slot = it;
    }
  } else if (warp == 1) {
    // ---- MMA issuer (rank 0) -----------------------------------------------------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = instr_desc_f16(kBf16, P_TILE_M, P_TILE_N);
      long long it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += pairs, ++local) {
        const int buf = local % kAccBufs;
        const int use = local / kAccBufs;
        if (use > 0 && !mbar_wait_bounded(&acc_empty[buf], (uint32_t)((use - 1) & 1), p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(buf * TMEM_COLS);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % P_STAGES);
          if (!mbar_wait_bounded(&full[s], (uint32_t)((it / P_STAGES) & 1), p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(a_tiles + s * P_A_BYTES);
          const uint64_t db = smem_desc_sw128(b_tiles + s * P_B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_f16_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(peer_addr(&empty[s], 0));
          umma_commit_pair(peer_addr(&empty[s], 1));
        }
        if (ok) {
          umma_commit_pair(peer_addr(&acc_full[buf], 0));
          umma_commit_pair(peer_addr(&acc_full[buf], 1));
        }
      }
    }
  } else {
    // ---- epilogue (both ranks): thread = accumulator row of this CTA --------------------
    const int q = warp & 3;
    constexpr int kCols = P_TILE_N * 4 / kEpiWarps;  // accumulator columns per epilogue warp
    const int c_begin = ((warp - 2) / 4) * kCols;
    const T* bias = reinterpret_cast<const T*>(p.bias);
    const int HD = p.H * p.D;
    const long long plane = (long long)p.T_out * p.D;
    const uint32_t empty0_a = peer_addr(&acc_empty[0], 0), empty0_b = peer_addr(&acc_empty[1], 0);
    int local = 0;
    for (int tile = pair; tile < n_tiles; tile += pairs, ++local) {
      const int buf = local % kAccBufs;
      const int n0 = pair_n0(tile, tiles_n, tiles_m), m0 = pair_m0(tile, tiles_n, tiles_m);
      const bool ready = mbar_wait_bounded(&acc_full[buf], (uint32_t)((local / kAccBufs) & 1), p.err);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int m = m0 + (int)rank * P_ROWS + q * 32 + lane;
      const bool row_ok = m < p.M;
      const int b = row_ok ? m / p.T : 0;
      const int t = row_ok ? m % p.T : 0;
      const long long slot = row_ok ? (p.slot_ids ? p.slot_ids[b] : b) : 0;
      T* out = reinterpret_cast<T*>(p.out) + slot * p.out_slot_stride + (long long)t * p.D;
#pragma unroll 1
      for (int c0 = c_begin; c0 < c_begin + kCols; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TMEM_COLS + c0), v);  // all lanes
        if (!row_ok) continue;
        store_row_chunk<T, 32>(v, n0 + c0, p.N, HD, p.H, p.D, plane, bias, out);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&acc_empty[buf]);
        else
          mbar_arrive_remote(buf ? empty0_b : empty0_a);
      }
    }
  }

  // ---- teardown ----------------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  cluster_barrier();  // both epilogues are done with TMEM; every MMA has completed
  if (rank == 0 && tid == 0) {
    // copies either producer issued that no MMA consumed (error paths only) land before
    // either CTA can leave: they all complete on rank 0's full barriers
    const long long mine = *issued_slot;
    long long theirs = 0;
    const uint32_t peer_issued = peer_addr(issued_slot, 1);
    asm volatile("ld.shared::cluster.b64 %0, [%1];" : "=l"(theirs) : "r"(peer_issued) : "memory");
    const long long upto = mine > theirs ? mine : theirs;
    for (long long k = upto - 1; k >= 0 && k >= upto - P_STAGES; --k)
      (void)mbar_wait_bounded(&full[k % P_STAGES], (uint32_t)((k / P_STAGES) & 1), nullptr);
  }
  cluster_barrier();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kAccBufs * TMEM_COLS);
}
}  // namespace proj

int cross_kv_project_launch(const void* enc_out, const void* w_kv, const void* b_kv, void* out,
                            const int32_t* slot_ids, int B, int T, int d_model, int L, int H, int D, int T_out,
                            int64_t out_slot_stride, int dtype, int* err, int sms, cudaStream_t st) {
  using namespace proj;
  if (sms < 1) sms = 1;
  const bool bf16 = dtype == SPD_BF16;
  const long long M = (long long)B * T, N = (long long)L * 2 * H * D;
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || (N % 8)) return SPD_ERR_UNSUPPORTED;
  Params p{};
  p.bias = b_kv; p.out = out; p.slot_ids = slot_ids;
  p.M = (int)M; p.N = (int)N; p.K = d_model; p.T = T; p.H = H; p.D = D; p.T_out = T_out;
  p.out_slot_stride = out_slot_stride; p.err = err;
  CUtensorMap ta, tb;
  // the CTA-pair form: 256 x 256 tiles on 2-CTA clusters, as many clusters as fit at once
  // the pair form wins from d_model 1024 up (large-v3, d 1280: 340 against 443 us per
  // request); at d 768 (Whisper-small: 12 K slices a tile) the one-CTA form is faster
  if (kProjPairs && sms >= 2 && d_model >= kPairMinK) {
    if (!make_map(&ta, enc_out, d_model, (int)M, P_ROWS, bf16) || !make_map(&tb, w_kv, d_model, (int)N, P_ROWS, bf16))
      return SPD_ERR_CUDA;
    auto launch_pair = [&](auto kfn) -> bool {
      if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM_BYTES) != cudaSuccess)
        return false;
      cudaLaunchConfig_t cfg = {};
      cfg.blockDim = dim3(kProjThreads);
      cfg.dynamicSmemBytes = P_SMEM_BYTES;
      cfg.stream = st;
      cfg.gridDim = dim3(2);
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg) != cudaSuccess || clusters < 1) return false;
      const long long tiles = ((N + P_TILE_N - 1) / P_TILE_N) * ((M + P_TILE_M - 1) / P_TILE_M);
      long long pairs = clusters < sms / 2 ? clusters : sms / 2;
      if (pairs > tiles) pairs = tiles;
      cfg.gridDim = dim3((unsigned)(2 * pairs));
      return cudaLaunchKernelEx(&cfg, kfn, ta, tb, p) == cudaSuccess;
    };
    const bool launched = bf16 ? launch_pair(cross_kv_project_pair_kernel<__nv_bfloat16>)
                               : launch_pair(cross_kv_project_pair_kernel<__half>);
    if (launched) return SPD_OK;
    (void)cudaGetLastError();  // the one-CTA form below
  }
  if (!make_map(&ta, enc_out, d_model, (int)M, BM, bf16) || !make_map(&tb, w_kv, d_model, (int)N, BN, bf16))
    return SPD_ERR_CUDA;
  const long long tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  dim3 grid((unsigned)(tiles < sms ? tiles : sms));  // persistent: at most one CTA per SM
  if (bf16) {
    auto k = cross_kv_project_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
      return SPD_ERR_CUDA;
    k<<<grid, kProjThreads, SMEM_BYTES, st>>>(ta, tb, p);
  } else {
    auto k = cross_kv_project_kernel<__half>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) != cudaSuccess)
      return SPD_ERR_CUDA;
    k<<<grid, kProjThreads, SMEM_BYTES, st>>>(ta, tb, p);
  }
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

}  // namespace spd
