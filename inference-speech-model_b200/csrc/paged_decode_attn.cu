// paged_decode_attn.cu — op (1): paged single-query decoder self-attention, with the
// new token's K/V write (op (3)) fused in front of it.
//
// Semantics follow the reference's direct paged kernel
// (scripts/evaluate_paging_variants.py:56-133): for each sequence b and head h,
//   out[b,h,:] = softmax_t( q[b,h,:]·K[t,h,:] * scale ) · V[t,h,:],  t in [0, ctx_b)
// where row t lives in pool block block_tables[b][t / block_size] at offset
// t % block_size.  The eager/graph paths of speech_serving/models.py:140-164 and
// :456-466 compute the same quantity over a contiguous or bucketed copy of the cache.
//
// B200 design (HBM-bound; no tensor cores):
// * A unit is one pool block of ALL heads: in the pool layout
//   [num_blocks][block_size][H][D] that is one contiguous run of block_size*H*D
//   elements, fetched with two 1-D bulk async copies (K and V; only the valid rows of a
//   sequence's last block) under an L2 evict-first policy.  A work item is chunk c of a
//   sequence: its units [c*kItemUnits, (c+1)*kItemUnits).
// * CTA g of the persistent grid starts on chunk g / B of sequence g % B: its producer
//   reads that sequence's length and block ids with plain loads, so the first copies go
//   out one round trip after the grid starts.  The lengths and the whole block table
//   (when it fits) arrive by bulk copy meanwhile; every other chunk is queued
//   (sequence-major) and handed out by a global atomic counter, one take ahead, so CTAs
//   whose data arrives early simply do more items and the kernel ends when the queue
//   drains.  The counter is reset by the last CTA to finish taking.
// * The producer streams units through an S-stage shared-memory ring (full mbarriers
//   complete on the copies' bytes, empty mbarriers collect one arrival per compute warp);
//   per-stage metadata says which sequence/block/item a stage holds; a stage with
//   sequence -1 ends the loop.  q (and, for the fused append, k_new/v_new) ride in the
//   stage of an item's first (last) unit.
// * Compute warp w owns heads [w*HPW, (w+1)*HPW) and never synchronises with the other
//   compute warps: it patches its own slice of an appended row; at the end of an item it
//   writes the output (an item covering the whole sequence) or a partial (m, l, acc) to
//   slot [b * chunks_per_sequence + c][h].
// * Split sequences are merged by a second, small kernel (one warp per (sequence, head))
//   launched with programmatic dependent launch: the streaming kernel signals
//   launch_dependents at its start, so the merge kernel's CTAs are already resident, have
//   read their sequence's length, and wait (griddepcontrol.wait) when the streaming
//   kernel ends; then one round of loads brings in every partial of the sequence.
// * q·k: 32/block_size lanes per row, q in registers (each score scaled by scale*log2 e), K
//   chunks read in a per-row rotated order so the 8 lanes of a shared-memory phase hit
//   distinct banks.  p·v: each lane owns one 16-byte chunk of a row.  Online softmax in
//   base 2; packed fp32x2 FMAs.
// * Every wait is bounded; a warp whose wait runs out records SPD_DEVERR_TIMEOUT, raises
//   the CTA's abort flag and leaves, and the others' bounded waits then run out too.
#include <type_traits>
#include <vector>

#include "spd_params.cuh"
#include "spd_trace.cuh"

// Timeline marks (trace builds only; see spd_trace.cuh).  Streaming kernel, per CTA:
// 0 entry, 6 griddepcontrol.wait returned, 2 first copy issued, 1 lengths scanned,
// 3 producer out of items, 4 first stage consumed (warp 0), 5 warp 0 done, 7 producer
// done, 8 last stage landed (seen by warp 0), 9 stages warp 0 processed (a count).
// Merge kernel, per CTA: 0 entry, 1 griddepcontrol.wait returned, 2 done.
SPD_TRACE_ARRAY
#define SPD_TRACE(point) SPD_TRACE_AT(0, point)
#define SPD_TRACE_MERGE(point) SPD_TRACE_AT(1, point)

namespace spd {

template <typename T>
struct Pair;
template <>
struct Pair<float> {
  static __device__ __forceinline__ float2 to_f2(const float* p) { return *reinterpret_cast<const float2*>(p); }
};
template <>
struct Pair<__half> {
  static __device__ __forceinline__ float2 to_f2(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
  }
};
template <>
struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_f2(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
};

// N consecutive elements (N even) -> N/2 float2, using the widest aligned vector load.
template <typename T, int N>
__device__ __forceinline__ void load_f2(const T* p, float2* out) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 16 / (int)sizeof(T)) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + i);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < 16 / (int)sizeof(T); k += 2) out[(i + k) / 2] = Pair<T>::to_f2(e + k);
    }
  } else if constexpr (BYTES % 8 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 8 / (int)sizeof(T)) {
      const uint2 v = *reinterpret_cast<const uint2*>(p + i);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < 8 / (int)sizeof(T); k += 2) out[(i + k) / 2] = Pair<T>::to_f2(e + k);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) out[i / 2] = Pair<T>::to_f2(p + i);
  }
}


template <typename T, int D, int BS>
struct PagedGeom {
  static constexpr int EB = sizeof(T);
  static constexpr int LPR = 32 / BS;                          // lanes per row for q·k
  static constexpr int DPL = D / LPR;                          // dims per lane for q·k
  static constexpr int CH = (DPL * EB >= 16) ? 16 / EB : DPL;  // elements per q·k chunk
  static constexpr int NCH = DPL / CH;                         // chunks per lane
  static constexpr int VE = 16 / EB;                           // elements per p·v chunk
  static constexpr int CPR = D / VE;                           // p·v chunks per row
  static constexpr int RG = 32 / CPR;                          // rows per p·v pass
  static constexpr int PVP = (BS + RG - 1) / RG;               // p·v passes per block
  static_assert(LPR * BS == 32 && DPL * LPR == D, "block_size must divide 32");
  static_assert(CPR * VE == D && RG * CPR == 32, "head_dim / dtype combination");
  static_assert((NCH & (NCH - 1)) == 0 && DPL % 2 == 0, "chunking");
};

// Per-stage metadata written by the producer before it arms the stage (two 16-byte words).
struct StageMeta {
  int b;        // sequence, or -1: no more work
  int nvalid;   // valid rows of this unit
  int slot;     // the item's partial slot: b * chunks_per_sequence + chunk
  int flags;    // kFirst | kLast | kAppend
  int phys;     // pool block of this unit
  int nchunks;  // items (chunks) of sequence b
  int pad0, pad1;
};
constexpr int kFirst = 1, kLast = 2, kAppend = 4;
constexpr int kPairThreads = 416;  // two-CTA form: up to 12 compute warps + the producer
#ifndef SPD_PAIR_MIN_SEQS
#define SPD_PAIR_MIN_SEQS 128
#endif
constexpr int kPairMinSeqs = SPD_PAIR_MIN_SEQS;  // batches at least this large use the two-CTA form

__device__ __forceinline__ int clamp_ctx(int c, int max_ctx) { return c > max_ctx ? max_ctx : (c > 0 ? c : 0); }

// floats per split partial row (acc[D], m, l, zeros): a whole number of 32-byte sectors
template <int D>
constexpr int kPartialRow = D + 8;
static_assert(kPartialRow<16> % 8 == 0 && kPartialRow<128> % 8 == 0, "sector-aligned partial rows");

// PAIR: the two-CTAs-per-SM form (at most 12 compute warps, registers capped for two
// resident CTAs, compact stages: the append rows are copied into the staged block).
template <typename T, int D, int BS, int HPW, bool PAIR>
__global__ void __launch_bounds__(PAIR ? kPairThreads : 544, PAIR ? 2 : 1)
    paged_decode_attn_kernel(const PagedParams p) {
  using Gm = PagedGeom<T, D, BS>;
  constexpr int LPR = Gm::LPR, DPL = Gm::DPL, CH = Gm::CH, NCH = Gm::NCH;
  constexpr int VE = Gm::VE, CPR = Gm::CPR, RG = Gm::RG, PVP = Gm::PVP;
  // q·k on the tensor cores (mma m16n8k16): 16-bit types, 16-row blocks, D of 64 or 128
  // (enough 8-element chunks per row for a conflict-free rotation over 8 rows)
  constexpr bool kMma = sizeof(T) == 2 && BS == 16 && (D == 64 || D == 128);
  static_assert(!kMma || (RG * PVP == BS && (8 % RG) == 0), "p·v row groups split at row 8");

  extern __shared__ __align__(128) unsigned char smem[];
  const int H = p.H, B = p.B, S = p.stages, MB = p.max_blocks;
  const int HD = H * D;
  const int NW = (H + HPW - 1) / HPW;  // compute warps; warp NW is the producer
  const int G = (int)gridDim.x;
  const int MC = (MB + kItemUnits - 1) / kItemUnits;  // chunks (items) of a sequence at most
  const size_t unit_elems = (size_t)BS * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- shared memory: ring | barriers | metadata | lengths | chunk prefix | table ----
  // K, V, q (and, in the single-CTA form, k_new / v_new rows for the fused append)
  const size_t stage_elems = 2 * unit_elems + (PAIR ? 1 : 3) * (size_t)HD;
  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + round_up((size_t)S * stage_elems * sizeof(T), 128));
  uint64_t* empty = full + S;
  uint64_t* setup = empty + S;
  StageMeta* meta = reinterpret_cast<StageMeta*>(setup + 2);  // 16-byte aligned
  int* flag = reinterpret_cast<int*>(meta + S);               // [0] abort, [1..3] spare
  int* ctx_s = flag + 4;                                      // [round4(B)] context lengths
  int* ip = ctx_s + ((B + 3) & ~3);                           // [B + 1] queued-chunk prefix
  int* tab_s = ip + ((B + 4) & ~3);                           // [B * MB] block table copy
  const bool tab_in_smem = p.table_in_smem != 0;

  int* next_item = p.work + 0;  // queue counter
  int* done_ctas = p.work + 1;  // CTAs that finished taking items
  const T* __restrict__ kpool = reinterpret_cast<const T*>(p.k_pool);
  const T* __restrict__ vpool = reinterpret_cast<const T*>(p.v_pool);
  T* __restrict__ out = reinterpret_cast<T*>(p.out);
  const T* __restrict__ qg = reinterpret_cast<const T*>(p.q);
  const bool append = p.k_new != nullptr;
  const int max_ctx = MB * BS;

  if (tid == 0) SPD_TRACE(0);
  // ---- 1. shared-memory set-up, while the previous kernel in the stream may still run --
  if (tid < 4) flag[tid] = 0;  // shared memory starts undefined
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    mbar_init(setup, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // Launched with programmatic dependent launch: this grid may become resident while the
  // previous kernel in the stream still runs, so every thread waits for it before reading
  // an input for use or writing an output.  Then the merge kernel that follows may get
  // resident early; it waits for this grid to finish (griddepcontrol.wait) before reading
  // anything.
  //
  // Before the wait, one compute warp only warms L2 (the producer goes straight to the
  // wait): it reads, bypassing L1, the length and block ids of this CTA's first chunk,
  // which the previous kernel may still be writing, and prefetches those blocks' K/V rows,
  // the lengths and the block table into L2.  A stale value only wastes a prefetch (block
  // ids are clamped into the pool); the rows are copied, and every input is read again,
  // after the wait.  So the DRAM fetch of every CTA's first chunk overlaps the previous
  // kernel's tail.
  if (warp == NW - 1 && lane == 0) {
    const int b0 = (int)blockIdx.x % B, c0 = (int)blockIdx.x / B;
    if (c0 < MC) {
      int phys[kItemUnits];
      const int ctx_raw = __ldcg(p.context_lens + b0);
#pragma unroll
      for (int u = 0; u < kItemUnits; ++u) {
        const int j = min(c0 * kItemUnits + u, MB - 1);
        phys[u] = __ldcg(p.block_tables + (size_t)b0 * MB + j);
      }
      const int ctx0 = clamp_ctx(ctx_raw, max_ctx);
      const uint32_t row_bytes = (uint32_t)(HD * (int)sizeof(T));
#pragma unroll
      for (int u = 0; u < kItemUnits; ++u) {
        const int j = c0 * kItemUnits + u;
        const int rows = min(BS, ctx0 - j * BS);
        if (j >= MB || rows <= 0) break;
        const int ph = phys[u] < 0 ? 0 : (phys[u] >= p.num_blocks ? p.num_blocks - 1 : phys[u]);
        bulk_prefetch_l2(kpool + (size_t)ph * unit_elems, (uint32_t)rows * row_bytes);
        bulk_prefetch_l2(vpool + (size_t)ph * unit_elems, (uint32_t)rows * row_bytes);
      }
    }
    if (blockIdx.x == 0) {
      if ((B * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.context_lens) & 15) == 0)
        bulk_prefetch_l2(p.context_lens, (uint32_t)B * 4u);
      if (tab_in_smem) bulk_prefetch_l2(p.block_tables, (uint32_t)B * MB * 4u);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) SPD_TRACE(6);

  // ---- 2. producer warp --------------------------------------------------------------
  // Work: chunk c of sequence b (blocks [c*kItemUnits, (c+1)*kItemUnits)) is one item.
  // CTA g starts on chunk g / B of sequence g % B, located with direct loads so that its
  // copies start one round trip after the wait; the other chunks form a queue (sequence-
  // major) handed out by a global counter once the lengths have arrived.
  if (warp == NW) {
    const uint64_t pol = l2_policy_evict_first();
    int s = 0;
    uint32_t ph = 0;
    long long n_issued = 0;
    bool alive = true;
    const uint32_t row_bytes = (uint32_t)(HD * (int)sizeof(T));
    // stages the unit j of item (b, chunk) (lane 0 only)
    auto issue_unit = [&](int b, int j, int ctx, int phys, int chunk, int nch, bool first, bool last) {
      if (n_issued >= S &&
          (*((volatile int*)&flag[0]) || !mbar_wait_bounded(&empty[s], ph ^ 1, p.err, p.wait_ns))) {
        flag[0] = 1;
        alive = false;
        return;
      }
      const int nblk = (ctx + BS - 1) / BS;
      const int nvalid = min(BS, ctx - j * BS);
      if (phys < 0 || phys >= p.num_blocks) {
        set_error(p.err, SPD_DEVERR_BLOCK_ID);
        phys = 0;
      }
      const bool app = append && (j == nblk - 1);
      meta[s] = StageMeta{b, nvalid, b * MC + chunk, (first ? kFirst : 0) | (last ? kLast : 0) | (app ? kAppend : 0),
                          phys, nch, 0, 0};
      const size_t off = (size_t)phys * unit_elems;
      T* dst = ring + (size_t)s * stage_elems;
      if constexpr (PAIR) {
        // compact stages: the new row (nvalid-1) comes from k_new / v_new straight into
        // its place, the pool supplies the rows before it
        const int npool = app ? nvalid - 1 : nvalid;
        const uint32_t bytes = (uint32_t)npool * row_bytes;
        mbar_arrive_expect_tx(&full[s], 2 * bytes + (first ? row_bytes : 0u) + (app ? 2 * row_bytes : 0u));
        if (npool > 0) {
          bulk_copy_g2s_hint(dst, kpool + off, bytes, &full[s], pol);
          bulk_copy_g2s_hint(dst + unit_elems, vpool + off, bytes, &full[s], pol);
        }
        if (first) bulk_copy_g2s(dst + 2 * unit_elems, qg + (size_t)b * HD, row_bytes, &full[s]);
        if (app) {
          bulk_copy_g2s(dst + (size_t)(nvalid - 1) * HD, reinterpret_cast<const T*>(p.k_new) + (size_t)b * HD,
                        row_bytes, &full[s]);
          bulk_copy_g2s(dst + unit_elems + (size_t)(nvalid - 1) * HD,
                        reinterpret_cast<const T*>(p.v_new) + (size_t)b * HD, row_bytes, &full[s]);
        }
      } else {
        const uint32_t bytes = (uint32_t)nvalid * row_bytes;
        mbar_arrive_expect_tx(&full[s], 2 * bytes + (first ? row_bytes : 0u) + (app ? 2 * row_bytes : 0u));
        bulk_copy_g2s_hint(dst, kpool + off, bytes, &full[s], pol);
        bulk_copy_g2s_hint(dst + unit_elems, vpool + off, bytes, &full[s], pol);
        if (first) bulk_copy_g2s(dst + 2 * unit_elems, qg + (size_t)b * HD, row_bytes, &full[s]);
        if (app) {
          bulk_copy_g2s(dst + 2 * unit_elems + HD, reinterpret_cast<const T*>(p.k_new) + (size_t)b * HD, row_bytes,
                        &full[s]);
          bulk_copy_g2s(dst + 2 * unit_elems + 2 * HD, reinterpret_cast<const T*>(p.v_new) + (size_t)b * HD,
                        row_bytes, &full[s]);
        }
      }
      if (n_issued == 0) SPD_TRACE(2);
      ++n_issued;
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
    };
    const bool ctx_bulk = ((B * 4) % 16 == 0) && ((reinterpret_cast<uintptr_t>(p.context_lens) & 15) == 0);
    int q = 0;
    if (lane == 0) {
      // lengths and table into shared memory, overlapping the first item's loads
      const uint32_t tx = (ctx_bulk ? (uint32_t)B * 4u : 0u) + (tab_in_smem ? (uint32_t)B * MB * 4u : 0u);
      if (tx) {
        mbar_arrive_expect_tx(setup, tx);
        if (ctx_bulk) bulk_copy_g2s(ctx_s, p.context_lens, (uint32_t)B * 4u, setup);
        if (tab_in_smem) bulk_copy_g2s(tab_s, p.block_tables, (uint32_t)B * MB * 4u, setup);
      } else {
        mbar_arrive(setup);
      }
      const int b0 = (int)blockIdx.x % B, c0 = (int)blockIdx.x / B;
      if (c0 < MC) {
        const int ctx0 = clamp_ctx(p.context_lens[b0], max_ctx);
        int ph0[kItemUnits];
#pragma unroll
        for (int u = 0; u < kItemUnits; ++u) {
          const int j = c0 * kItemUnits + u;
          ph0[u] = j < MB ? p.block_tables[(size_t)b0 * MB + j] : 0;
        }
        const int nblk0 = (ctx0 + BS - 1) / BS;
        const int nch0 = (nblk0 + kItemUnits - 1) / kItemUnits;
        if (c0 < nch0) {
          const int j0 = c0 * kItemUnits, j1 = min(j0 + kItemUnits, nblk0);
#pragma unroll
          for (int u = 0; u < kItemUnits; ++u)
            if (j0 + u < j1 && alive) issue_unit(b0, j0 + u, ctx0, ph0[u], c0, nch0, u == 0, j0 + u == j1 - 1);
        }
      }
      q = atomicAdd(next_item, 1);  // first queue take, in flight during the scan
    }
    __syncwarp();
    // lengths: clamp, chunks per sequence, and the prefix of each sequence's queued chunks
    // (its chunks minus the ones CTAs started on)
    if (!mbar_wait_bounded(setup, 0, p.err, p.wait_ns)) flag[0] = 1;
    if (!ctx_bulk)
      for (int i = lane; i < B; i += 32) ctx_s[i] = p.context_lens[i];
    __syncwarp();
    {
      int carry = 0;
      for (int base = 0; base < B; base += 32) {
        const int i = base + lane;
        int v = 0;
        if (i < B) {
          const int c0 = ctx_s[i];
          if (c0 > max_ctx) set_error(p.err, SPD_DEVERR_LENGTH);
          const int c = clamp_ctx(c0, max_ctx);
          ctx_s[i] = c;
          const int nch = ((c + BS - 1) / BS + kItemUnits - 1) / kItemUnits;
          const int started = i < G ? min((G - 1 - i) / B + 1, nch) : 0;
          v = nch - started;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += n;
        }
        if (i < B) ip[i + 1] = v + carry;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
      if (lane == 0) ip[0] = 0;
    }
    __syncwarp();
    if (lane == 0) SPD_TRACE(1);
    // sequences with nothing to attend to get zeros (sequence b by CTA b % G)
    for (int b = blockIdx.x; b < B; b += G)
      if (ctx_s[b] == 0)
        for (int i = lane; i < HD; i += 32) out[(size_t)b * HD + i] = Elem<T>::from_f(0.f);
    if (lane == 0) {
      const int n_queue = ip[B];
      alive = alive && !flag[0];
      while (alive && q < n_queue) {
        const int nxt = atomicAdd(next_item, 1);  // next take, in flight meanwhile
        const int b = upper_index_i32(ip, B, q);
        const int ctx = ctx_s[b];
        const int nblk = (ctx + BS - 1) / BS;
        const int nch = (nblk + kItemUnits - 1) / kItemUnits;
        const int started = b < G ? min((G - 1 - b) / B + 1, nch) : 0;
        const int c = started + (q - ip[b]);
        const int j0 = c * kItemUnits, j1 = min(j0 + kItemUnits, nblk);
        for (int j = j0; j < j1 && alive; ++j) {
          const int phys = tab_in_smem ? tab_s[b * MB + j] : p.block_tables[(size_t)b * MB + j];
          issue_unit(b, j, ctx, phys, c, nch, j == j0, j == j1 - 1);
        }
        q = nxt;
      }
      SPD_TRACE(3);
      // end-of-work stage for the compute warps
      if (alive && n_issued >= S && !mbar_wait_bounded(&empty[s], ph ^ 1, p.err, p.wait_ns)) alive = false;
      if (alive) {
        meta[s] = StageMeta{-1, 0, 0, 0, 0, 0, 0, 0};
        mbar_arrive(&full[s]);
      } else {
        flag[0] = 1;
      }
      // This CTA takes no more items; the last CTA to get here re-arms the counter for
      // the next launch (every CTA's final take has already happened).
      __threadfence();
      if (atomicAdd(done_ctas, 1) == G - 1) {
        *((volatile int*)next_item) = 0;
        *((volatile int*)done_ctas) = 0;
        __threadfence();
      }
      // After an abort, copies still in flight land before this CTA's shared memory is
      // released (without an abort the compute warps consumed every one of them).
      if (!alive) {
        for (int k = 0; k < S && k < n_issued; ++k) {
          const long long u = n_issued - 1 - k;
          (void)mbar_wait_bounded(&full[u % S], (uint32_t)((u / S) & 1), nullptr);
        }
        (void)mbar_wait_bounded(setup, 0, nullptr);  // the lengths / table copies
      }
      SPD_TRACE(7);
    }
    return;
  }

  // ---- 3. compute warps (independent of each other) ----------------------------------
  const int r = lane / LPR;    // q·k row of this lane
  const int sub = lane % LPR;  // which DPL-slice of the row
  const int rot = r & (NCH - 1);
  const int cidx = lane % CPR;  // p·v chunk of this lane
  const int rg = lane / CPR;    // p·v row group
  // tensor-core q·k (16-bit types, 16-row blocks, D = 64 or 128): fragment coordinates
  const int fg = lane >> 2, fc = lane & 3;

  float2 qr[HPW][kMma ? 1 : DPL / 2];
  uint32_t qb[HPW][kMma ? D / 8 : 1];
  float m[HPW], l[HPW];
  float2 acc[HPW][VE / 2];
  int s = 0;
  uint32_t ph = 0;
  bool traced = false;
  int n_stages = 0;
  for (;;) {
    if (*((volatile int*)&flag[0]) || !mbar_wait_bounded(&full[s], ph, p.err, p.wait_ns)) {
      flag[0] = 1;
      return;
    }
    const StageMeta mt = meta[s];
    if (mt.b < 0) break;
    if (tid == 0) {
      if (!traced) SPD_TRACE(4);
      traced = true;
      SPD_TRACE(8);
      ++n_stages;
    }
    const int b = mt.b;
    const int nvalid = mt.nvalid;
    T* Ks = ring + (size_t)s * stage_elems;
    T* Vs = Ks + unit_elems;
    const T* Qs = Vs + unit_elems;

    if (mt.flags & kFirst) {
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        m[k] = -INFINITY;
        l[k] = 0.f;
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) acc[k][i] = make_float2(0.f, 0.f);
        if (h < H) {
          if constexpr (kMma) {
            // B fragments of q: column n of k-step j holds q's 8-element chunks
            // (2j + n) and (2j + 1 + n) mod D/8 (see the q·k comment below)
            const T* qrow = Qs + h * D;
#pragma unroll
            for (int j = 0; j < D / 16; ++j) {
              qb[k][2 * j] = lds_u32(qrow + ((2 * j + fg) & (D / 8 - 1)) * 8 + 2 * fc);
              qb[k][2 * j + 1] = lds_u32(qrow + ((2 * j + 1 + fg) & (D / 8 - 1)) * 8 + 2 * fc);
            }
          } else {
            const T* qrow = Qs + h * D + sub * DPL;
#pragma unroll
            for (int cc = 0; cc < NCH; ++cc) {
              const int ci = (cc + rot) & (NCH - 1);
              load_f2<T, CH>(qrow + ci * CH, &qr[k][cc * CH / 2]);  // the score is scaled instead
            }
          }
        }
      }
    }

    if (mt.flags & kAppend) {
      // op (3) fused: the new token is row nvalid-1 of the last block; this warp writes
      // its own heads' slice into the stage (so its q·k sees it) and into the pool.
      const size_t blk = (size_t)mt.phys * unit_elems;
      const size_t row_off = (size_t)(nvalid - 1) * HD;
      constexpr int VEC = 16 / sizeof(T);
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        if (h >= H) break;
        for (int i = lane * VEC; i < D; i += 32 * VEC) {
          const size_t e = row_off + (size_t)h * D + i;
          if constexpr (PAIR) {  // the new row arrived in its place in the staged block
            *reinterpret_cast<uint4*>(const_cast<T*>(kpool) + blk + e) = *reinterpret_cast<const uint4*>(Ks + e);
            *reinterpret_cast<uint4*>(const_cast<T*>(vpool) + blk + e) = *reinterpret_cast<const uint4*>(Vs + e);
          } else {  // fill the new row's place in the staged block, and the pool
            const uint4 kv = *reinterpret_cast<const uint4*>(Qs + HD + h * D + i);
            const uint4 vv = *reinterpret_cast<const uint4*>(Qs + 2 * HD + h * D + i);
            *reinterpret_cast<uint4*>(Ks + e) = kv;
            *reinterpret_cast<uint4*>(Vs + e) = vv;
            *reinterpret_cast<uint4*>(const_cast<T*>(kpool) + blk + e) = kv;
            *reinterpret_cast<uint4*>(const_cast<T*>(vpool) + blk + e) = vv;
          }
        }
      }
      if constexpr (!PAIR) fence_proxy_async_smem();  // generic writes before the next bulk copy into this stage
      __syncwarp();
    }

    // One head of one block; FULL: all BS rows valid (every block but a sequence's last),
    // compiled without the per-row checks.
    auto head_block = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        if (h >= H) continue;
        const T* Kh = Ks + h * D;
        const T* Vh = Vs + h * D;
        if constexpr (kMma) {
          // q·k of the block's 16 rows as one m16n8k16 MMA chain: A = the K rows (row m,
          // D in k-steps of 16), B = q.  Every 8-element chunk of a row sits at the same
          // bank offset in every row (the row stride is a multiple of 128 bytes), so row
          // m reads its chunks in an order rotated by m mod 8 — its k-step j covers chunks
          // (2j + m) and (2j + 1 + m) mod D/8 — and B column n carries q's chunks in the
          // order rotated by n.  The 8 rows of a fragment load then hit 8 different bank
          // groups, and D[m][m mod 8] is row m's full dot product: row g's and row g+8's
          // scores end up in lane 4g + g/2 (element g & 1 of each row pair).
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          const T* k0 = Kh + (size_t)fg * HD;
          const T* k1 = k0 + (size_t)8 * HD;
#pragma unroll
          for (int j = 0; j < D / 16; ++j) {
            const int lo = ((2 * j + fg) & (D / 8 - 1)) * 8 + 2 * fc;
            const int hi = ((2 * j + 1 + fg) & (D / 8 - 1)) * 8 + 2 * fc;
            mma_16816<T>(d, lds_u32(k0 + lo), lds_u32(k1 + lo), lds_u32(k0 + hi), lds_u32(k1 + hi), qb[k][2 * j],
                         qb[k][2 * j + 1]);
          }
          const bool owner = fc == (fg >> 1);
          const float sa = (fg & 1) ? d[1] : d[0];  // row fg
          const float sb = (fg & 1) ? d[3] : d[2];  // row fg + 8
          const float s0 = (owner && (FULL || fg < nvalid)) ? sa * p.scale_log2 : -INFINITY;
          const float s1 = (owner && (FULL || fg + 8 < nvalid)) ? sb * p.scale_log2 : -INFINITY;
          const float mnew = fmaxf(m[k], warp_max_redux(fmaxf(s0, s1)));
          const float alpha = ex2_approx(m[k] - mnew);
          const float p0 = ex2_approx(s0 - mnew), p1 = ex2_approx(s1 - mnew);  // 0 off the owners
          l[k] = l[k] * alpha + (p0 + p1);
          m[k] = mnew;
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
          for (int i = 0; i < VE / 2; ++i) acc[k][i] = __fmul2_rn(acc[k][i], a2);
#pragma unroll
          for (int ps = 0; ps < PVP; ++ps) {
            const int rr = ps * RG + rg;
            const int src = 4 * (rr & 7) + ((rr & 7) >> 1);  // the lane holding row rr's weight
            const float prr = __shfl_sync(0xffffffffu, ps * RG < 8 ? p0 : p1, src);
            if ((FULL && rr < BS) || rr < nvalid) {
              float2 vv[VE / 2];
              load_f2<T, VE>(Vh + (size_t)rr * HD + cidx * VE, vv);
              const float2 p2 = make_float2(prr, prr);
#pragma unroll
              for (int i = 0; i < VE / 2; ++i) acc[k][i] = __ffma2_rn(p2, vv[i], acc[k][i]);
            }
          }
          continue;
        }
        const bool rv = FULL || r < nvalid;
        float sc = 0.f;
        if (rv) {
          const T* krow = Kh + (size_t)r * HD + sub * DPL;
          float2 dot = make_float2(0.f, 0.f);
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            const int ci = (cc + rot) & (NCH - 1);
            float2 kv[CH / 2];
            load_f2<T, CH>(krow + ci * CH, kv);
#pragma unroll
            for (int e = 0; e < CH / 2; ++e) dot = __ffma2_rn(qr[k][cc * CH / 2 + e], kv[e], dot);
          }
          sc = dot.x + dot.y;
        }
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        sc = rv ? sc * p.scale_log2 : -INFINITY;
        const float mnew = fmaxf(m[k], warp_max(sc));
        const float alpha = ex2_approx(m[k] - mnew);
        const float pr = rv ? ex2_approx(sc - mnew) : 0.f;
        l[k] = l[k] * alpha + (sub == 0 ? pr : 0.f);
        m[k] = mnew;
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) acc[k][i] = __fmul2_rn(acc[k][i], a2);
#pragma unroll
        for (int ps = 0; ps < PVP; ++ps) {
          const int rr = ps * RG + rg;
          const float prr = __shfl_sync(0xffffffffu, pr, (rr < BS ? rr : 0) * LPR);
          if ((FULL && rr < BS) || rr < nvalid) {
            float2 vv[VE / 2];
            load_f2<T, VE>(Vh + (size_t)rr * HD + cidx * VE, vv);
            const float2 p2 = make_float2(prr, prr);
#pragma unroll
            for (int i = 0; i < VE / 2; ++i) acc[k][i] = __ffma2_rn(p2, vv[i], acc[k][i]);
          }
        }
      }
    };
    if (nvalid == BS)
      head_block(std::true_type{});
    else
      head_block(std::false_type{});
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }

    if (!(mt.flags & kLast)) continue;
    // ---- item end: the output, or a partial for the merge kernel --------------------------
    const int nitems = mt.nchunks;
#pragma unroll
    for (int k = 0; k < HPW; ++k) {
      const int h = warp * HPW + k;
      if (h >= H) continue;
      const float ltot = warp_sum(l[k]);
#pragma unroll
      for (int o = CPR; o < 32; o <<= 1)
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) {
          acc[k][i].x += __shfl_xor_sync(0xffffffffu, acc[k][i].x, o);
          acc[k][i].y += __shfl_xor_sync(0xffffffffu, acc[k][i].y, o);
        }
      if (nitems == 1) {
        if (rg == 0) {
          const float inv = 1.f / ltot;
          T* orow = out + ((size_t)b * H + h) * D + cidx * VE;
#pragma unroll
          for (int i = 0; i < VE / 2; ++i) {
            orow[2 * i] = Elem<T>::from_f(acc[k][i].x * inv);
            orow[2 * i + 1] = Elem<T>::from_f(acc[k][i].y * inv);
          }
        }
        continue;
      }
      // a partial row: acc[D], then (m, l) and zeros filling the last 32-byte sector; kept
      // in L2 for the merge kernel
      float* slot = p.partials + ((size_t)mt.slot * H + h) * kPartialRow<D>;
      const uint64_t keep = l2_policy_evict_last();
      if (rg == 0) {
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) st_global_hint(slot + cidx * VE + 2 * i, acc[k][i], keep);
      }
      if (lane == 0) {
        st_global_hint(slot + D, make_float4(m[k], ltot, 0.f, 0.f), keep);
        st_global_hint(slot + D + 4, make_float4(0.f, 0.f, 0.f, 0.f), keep);
      }
    }
  }
  if (tid == 0) {
    SPD_TRACE(5);
    SPD_TRACE_VALUE(0, 9, n_stages);
  }
  (void)n_stages;
}

// ------------------------------------------------------------------ merge kernel
// One warp per (sequence, head) of a sequence that spans more than one item.  Launched
// with programmatic dependent launch right behind the streaming kernel.  The sequence's
// length is read while the streaming kernel still runs: the streaming kernel never writes
// it, and it triggers this launch only after its own griddepcontrol.wait, so everything
// written before it is final.  The partials of sequence b sit at slots
// [b * chunks_per_sequence, + its chunks); after griddepcontrol.wait all of them are
// loaded in one round trip (lane = item for (m, l); all items' acc before any is used).
template <typename T, int D, int BS>
__global__ void __launch_bounds__(128) paged_merge_kernel(const PagedParams p) {
  constexpr int DL = (D + 31) / 32;             // acc elements per lane (two-pass path)
  constexpr int EPL = D >= 64 ? D / 32 : 2;      // acc elements per lane (register path)
  using V = std::conditional_t<EPL == 4, float4, float2>;
  static_assert(EPL == 2 || EPL == 4, "head_dim");
  constexpr int MAXI = 16;  // items per sequence held in registers (a 448-token context has 14)
  const int lane = threadIdx.x & 31;
  const long long pair = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const bool live = pair < (long long)p.B * p.H;
  const int b = live ? (int)(pair / p.H) : 0, h = live ? (int)(pair % p.H) : 0;
  const int max_ctx = p.max_blocks * BS;
  const int MC = (p.max_blocks + kItemUnits - 1) / kItemUnits;
  const int ctx_b = live ? clamp_ctx(p.context_lens[b], max_ctx) : 0;
  const int nitems = ((ctx_b + BS - 1) / BS + kItemUnits - 1) / kItemUnits;
  if (threadIdx.x == 0) SPD_TRACE_MERGE(0);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the streaming kernel has finished
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) SPD_TRACE_MERGE(1);
  if (!live || nitems <= 1) return;  // written by the streaming kernel (or zero)
  const float* base = p.partials + ((size_t)b * MC * p.H + h) * kPartialRow<D>;
  const size_t stride = (size_t)p.H * kPartialRow<D>;  // next item, same head
  T* orow = reinterpret_cast<T*>(p.out) + ((size_t)b * p.H + h) * D;
  if (nitems <= MAXI) {
    // lane l holds elements [l*EPL, (l+1)*EPL) of every item's acc: one vector load per item
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < nitems) ml = __ldcg(reinterpret_cast<const float2*>(base + lane * stride + D));
    const bool hold = lane < D / EPL;
    V a[MAXI];
#pragma unroll
    for (int it = 0; it < MAXI; ++it)
      a[it] = (it < nitems && hold) ? __ldcg(reinterpret_cast<const V*>(base + it * stride) + lane) : V{};
    const float M = warp_max(ml.x);
    const float w = lane < nitems ? exp2f(ml.x - M) : 0.f;
    const float inv = 1.f / warp_sum(ml.y * w);
    V o{};
#pragma unroll
    for (int it = 0; it < MAXI; ++it) {
      const float wi = __shfl_sync(0xffffffffu, w, it);
      o.x = fmaf(wi, a[it].x, o.x);
      o.y = fmaf(wi, a[it].y, o.y);
      if constexpr (EPL == 4) {
        o.z = fmaf(wi, a[it].z, o.z);
        o.w = fmaf(wi, a[it].w, o.w);
      }
    }
    if (hold) {
      T* dst = orow + lane * EPL;
      dst[0] = Elem<T>::from_f(o.x * inv);
      dst[1] = Elem<T>::from_f(o.y * inv);
      if constexpr (EPL == 4) {
        dst[2] = Elem<T>::from_f(o.z * inv);
        dst[3] = Elem<T>::from_f(o.w * inv);
      }
    }
    if ((threadIdx.x & 31) == 0) SPD_TRACE_MERGE(2);
    return;
  }
  // long sequences: two passes over the items
  float M = -INFINITY;
  for (int it = lane; it < nitems; it += 32) M = fmaxf(M, __ldcg(base + it * stride + D));
  M = warp_max(M);
  float L = 0.f;
  for (int it = lane; it < nitems; it += 32)
    L += __ldcg(base + it * stride + D + 1) * exp2f(__ldcg(base + it * stride + D) - M);
  const float inv = 1.f / warp_sum(L);
#pragma unroll
  for (int e = 0; e < DL; ++e) {
    const int d = lane + 32 * e;
    if (d >= D) break;
    float o = 0.f;
    for (int it = 0; it < nitems; ++it)
      o = fmaf(exp2f(__ldcg(base + it * stride + D) - M), __ldcg(base + it * stride + d), o);
    orow[d] = Elem<T>::from_f(o * inv);
  }
}

// ------------------------------------------------------------------ host launcher
template <typename T, int D, int BS>
static int launch_merge(const PagedParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((long long)p.B * p.H + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, paged_merge_kernel<T, D, BS>, p) == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

template <typename T, int D, int BS, int HPW, bool PAIR>
static int launch_paged(const PagedParams& base, int device_sms, cudaStream_t stream) {
  PagedParams p = base;
  const int nw = (p.H + HPW - 1) / HPW;
  const int threads = (nw + 1) * 32;  // compute warps + producer warp
  if (PAIR && threads > kPairThreads) return SPD_ERR_UNSUPPORTED;
  const size_t stage_bytes = ((size_t)2 * BS + (PAIR ? 1 : 3)) * p.H * D * sizeof(T);
  const size_t tab_bytes = (size_t)p.B * p.max_blocks * 4;
  p.table_in_smem = (tab_bytes <= kTableSmemMax && tab_bytes % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(p.block_tables) & 15) == 0)
                        ? 1
                        : 0;
  const size_t fixed = 16 * 8 /*barriers*/ + 32 * 8 /*meta*/ + 16 + 4 * ((size_t)p.B + 4) * 2 +
                       (p.table_in_smem ? tab_bytes : 0) + 256;
  // Ring depth: up to ~216 KB per CTA (one CTA per SM at the Whisper shapes; the
  // producer warp keeps every stage in flight), at least two stages.
  const size_t budget = (PAIR ? 112 : 216) * 1024;
  int S = (int)((budget > fixed ? budget - fixed : 0) / stage_bytes);
  if (S < 2 && 2 * stage_bytes + fixed <= 227 * 1024) S = 2;
  S = S < 1 ? 1 : (S > 8 ? 8 : S);
  p.stages = S;
  const size_t smem = round_up((size_t)S * stage_bytes, 128) + 16 * ((size_t)S * 2 + 2) + 32 * (size_t)S + 16 +
                      4 * ((((size_t)p.B + 3) & ~(size_t)3) + (((size_t)p.B + 4) & ~(size_t)3)) +
                      (p.table_in_smem ? tab_bytes : 0);
  if (smem > (PAIR ? 113 : 227) * 1024) return SPD_ERR_UNSUPPORTED;
  auto kfn = paged_decode_attn_kernel<T, D, BS, HPW, PAIR>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SPD_ERR_CUDA;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, threads, smem) != cudaSuccess || occ < 1)
    return SPD_ERR_CUDA;
  if (PAIR && occ < 2) return SPD_ERR_UNSUPPORTED;
  if (occ > kMaxCtasPerSm) occ = kMaxCtasPerSm;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(device_sms * occ));
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kfn, p) != cudaSuccess) return SPD_ERR_CUDA;
  return launch_merge<T, D, BS>(p, stream);
}

template <typename T, int D, int BS>
static int launch_paged_bs(const PagedParams& p, int sms, cudaStream_t st) {
  if (p.H > 16) return launch_paged<T, D, BS, 2, false>(p, sms, st);
  // Large batches: two CTAs per SM (twice the compute warps to hide the per-block
  // latency, more bytes in flight).  Small ones keep one CTA per SM: with fewer items per
  // CTA the per-CTA set-up costs more than the extra warps save.
  if (p.B >= kPairMinSeqs) {
    const int rc = launch_paged<T, D, BS, 1, true>(p, sms, st);
    if (rc != SPD_ERR_UNSUPPORTED) return rc;
  }
  return launch_paged<T, D, BS, 1, false>(p, sms, st);
}

template <typename T, int D>
static int dispatch_bs(const PagedParams& p, int bs, int sms, cudaStream_t st) {
  switch (bs) {
    case 8: return launch_paged_bs<T, D, 8>(p, sms, st);
    case 16: return launch_paged_bs<T, D, 16>(p, sms, st);
    case 32:
      if constexpr (D <= 64) return launch_paged_bs<T, D, 32>(p, sms, st);
      return SPD_ERR_UNSUPPORTED;
    default: return SPD_ERR_UNSUPPORTED;
  }
}

template <typename T>
static int dispatch_d(const PagedParams& p, int D, int bs, int sms, cudaStream_t st) {
  switch (D) {
    case 16: return dispatch_bs<T, 16>(p, bs, sms, st);
    case 32: return dispatch_bs<T, 32>(p, bs, sms, st);
    case 64: return dispatch_bs<T, 64>(p, bs, sms, st);
    case 128: return dispatch_bs<T, 128>(p, bs, sms, st);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

int paged_decode_attn_launch(const PagedParams& p, int dtype, int D, int bs, int sms, cudaStream_t st) {
  switch (dtype) {
    case SPD_F32: return dispatch_d<float>(p, D, bs, sms, st);
    case SPD_F16: return dispatch_d<__half>(p, D, bs, sms, st);
    case SPD_BF16: return dispatch_d<__nv_bfloat16>(p, D, bs, sms, st);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

}  // namespace spd

#ifdef SPD_TRACE_BUILD
// Trace builds only: copies the last launch's marks, [kernel][CTA][point] as unsigned
// 64-bit %globaltimer values (0 where a mark was not reached), into `host` (synchronous).
extern "C" int spd_trace_fetch_paged(unsigned long long* host, size_t count) {
  const size_t n = (size_t)spd::kTraceKernels * spd::kTraceCtas * spd::kTracePoints;
  if (!host || count < n) return SPD_ERR_INVALID_ARG;
  if (cudaMemcpyFromSymbol(host, spd::g_trace, n * sizeof(unsigned long long)) != cudaSuccess) return SPD_ERR_CUDA;
  std::vector<unsigned long long> zero(n, 0ull);
  return cudaMemcpyToSymbol(spd::g_trace, zero.data(), n * sizeof(unsigned long long)) == cudaSuccess ? SPD_OK
                                                                                                     : SPD_ERR_CUDA;
}
#endif
