// cross_attn.cu — op (2): single-query cross-attention over contiguous encoder K/V.
//
// Semantics follow speech_serving/models.py:167-203 (eager) and :468-479 (graph step):
//   out[b,h,:] = softmax_t( q[b,h,:]·K[b,h,t,:] * scale ) · V[b,h,t,:],  t < valid_b
// Positions at or beyond valid_b are excluded, which equals the reference's bool mask
// filled with finfo.min (models.py:196-197) and its additive -10000 fp16 mask
// (graph_decode_buffers.py:529): both drive exp() of those scores to exactly 0.
//
// B200 design (HBM-bound):
// * A unit is a chunk of C consecutive positions of one (b, h) pair — C*D contiguous
//   elements of K and of V — fetched with two 1-D bulk async copies (only valid rows)
//   under an L2 evict-first policy.  A work item is up to `item_units` consecutive units
//   of one pair (so a pair has at most kCrossMaxItems items).
// * Items are handed out dynamically: CTA g of the persistent grid starts on item g and
//   its producer warp takes further items from a global atomic counter, one take ahead, so
//   CTAs whose data arrives early do more items and no CTA straggles behind a static
//   share.  The last CTA to finish taking resets the counter (graph-safe).
// * Within a CTA the compute warps split each unit's rows; at an item's end their
//   online-softmax states are merged in shared memory.  An item that covers its whole pair
//   writes the output; otherwise it writes a partial (m, l, acc) to slot [item], stored
//   evict-last, and a second kernel, launched with programmatic dependent launch, merges
//   the pair's partials (one warp per pair, all partials in one round of loads).
#include <type_traits>

#include "spd_params.cuh"

namespace spd {

constexpr int kCrossComputeBarrier = 1;  // named barrier among compute warps
constexpr int kCrossFirst = 1, kCrossLast = 2;

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <typename T, int D>
struct CrossGeom {
  static constexpr int EB = sizeof(T);
  static constexpr int NW = 8;                                   // warps per CTA
  static constexpr int LPR = (D * EB / 64) > 1 ? (D * EB / 64) : 1;  // lanes per row (64 B each)
  static constexpr int RPP = 32 / LPR;                           // rows per warp pass
  static constexpr int DPL = D / LPR;
  static constexpr int CH = (DPL * EB >= 16) ? 16 / EB : DPL;
  static constexpr int NCH = DPL / CH;
  static constexpr int PASSES = (16384 / (NW * RPP * D * EB)) > 1 ? (16384 / (NW * RPP * D * EB)) : 1;
  static constexpr int C = NW * RPP * PASSES;                    // rows per unit
  static constexpr int PVL = D >= 32 ? 32 : D;
  static constexpr int PRG = 32 / PVL;
  static constexpr int DPV = D / PVL;
};

// Per-stage metadata written by the producer before it arms the stage.
struct CrossStage {
  int b;      // sequence, or -1: no more work
  int h;      // head
  int j;      // unit within the pair
  int item;   // item of the pair (0, 1, ...)
  int flags;  // kCrossFirst | kCrossLast
  int pad0, pad1, pad2;
};

__device__ __forceinline__ int clamp_valid(int v, int t_max) { return v > t_max ? t_max : (v > 0 ? v : 0); }

template <typename T, int D>
__global__ void __launch_bounds__(288) cross_attn_kernel(const CrossParams p) {
  using Gm = CrossGeom<T, D>;
  constexpr int NW = Gm::NW, LPR = Gm::LPR, RPP = Gm::RPP, DPL = Gm::DPL, CH = Gm::CH;
  constexpr int NCH = Gm::NCH, PASSES = Gm::PASSES, C = Gm::C;
  constexpr int PVL = Gm::PVL, PRG = Gm::PRG, DPV = Gm::DPV;
  constexpr int NCT = NW * 32;  // compute threads; warp NW is the producer

  extern __shared__ __align__(128) unsigned char smem[];
  const int H = p.H, B = p.B, S = p.stages, N = p.item_units;
  const size_t unit_elems = (size_t)C * D;
  const size_t stage_elems = 2 * unit_elems + D;  // K chunk, V chunk, q row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + round_up((size_t)S * stage_elems * sizeof(T), 128));
  uint64_t* empty = full + S;
  CrossStage* meta = reinterpret_cast<CrossStage*>(empty + S);  // [S]
  float* merge = reinterpret_cast<float*>(meta + S);             // [NW][D + 2]
  int* ip = reinterpret_cast<int*>(merge + NW * (D + 2));        // [B + 1] item prefix over sequences
  int* qp = ip + B + 1;                                          // [B + 1] queued-item prefix
  int* nch_s = qp + B + 1;                                       // [B] units per pair
  int* val_s = nch_s + B;                                        // [B] clamped valid length
  int* flag = val_s + B;                                         // [0] abort

  int* next_item = p.work + 0;  // item counter
  int* done_ctas = p.work + 1;  // CTAs that finished taking
  const T* __restrict__ kg = reinterpret_cast<const T*>(p.k);
  const T* __restrict__ vg = reinterpret_cast<const T*>(p.v);
  const T* __restrict__ qg = reinterpret_cast<const T*>(p.q);
  T* __restrict__ out = reinterpret_cast<T*>(p.out);

  // the merge kernel behind this one may get resident now; it waits for this grid to end
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_barrier_init();
    flag[0] = 0;
  }
  __syncthreads();

  // producer state (lane 0 of warp NW)
  const int G = (int)gridDim.x, P = B * H;
  int s_p = 0;
  uint32_t ph_p = 0;
  long long n_issued = 0;
  bool alive = true;
  const uint64_t pol = l2_policy_evict_first();
  // stages the units of item k of pair (b, h): units [k*N, min((k+1)*N, nch)) of valid length v
  auto issue_item = [&](int b, int h, int k, int v, int nch) {
    const int j0 = k * N, j1 = min(j0 + N, nch);
    for (int j = j0; j < j1; ++j) {
      if (n_issued >= S &&
          (*((volatile int*)&flag[0]) || !mbar_wait_bounded(&empty[s_p], ph_p ^ 1, p.err, p.wait_ns))) {
        flag[0] = 1;
        alive = false;
        return;
      }
      const int nrows = min(C, v - j * C);
      const size_t src = (size_t)b * p.kv_batch_stride + (size_t)h * p.kv_head_stride + (size_t)j * C * D;
      const uint32_t bytes = (uint32_t)(nrows * D * (int)sizeof(T));
      const bool first = (j == j0);
      const uint32_t qbytes = first ? (uint32_t)(D * sizeof(T)) : 0u;
      meta[s_p] = CrossStage{b, h, j, k, (first ? kCrossFirst : 0) | (j == j1 - 1 ? kCrossLast : 0), 0, 0, 0};
      T* dst = ring + (size_t)s_p * stage_elems;
      mbar_arrive_expect_tx(&full[s_p], 2 * bytes + qbytes);
      bulk_copy_g2s_hint(dst, kg + src, bytes, &full[s_p], pol);
      bulk_copy_g2s_hint(dst + unit_elems, vg + src, bytes, &full[s_p], pol);
      if (first) bulk_copy_g2s(dst + 2 * unit_elems, qg + ((size_t)b * H + h) * D, qbytes, &full[s_p]);
      ++n_issued;
      if (++s_p == S) {
        s_p = 0;
        ph_p ^= 1;
      }
    }
  };
  // CTA g starts on item 0 of pair g, located with one direct load: its copies go out while
  // the lengths are scanned.  Before the compute warps run nothing frees a stage, so an
  // item with more units than the ring has stages waits until after the scan.
  int v0 = 0, nch0 = 0;
  if (warp == NW && lane == 0 && (int)blockIdx.x < P) {
    v0 = clamp_valid(p.valid_lens[(int)blockIdx.x / H], p.T_max);
    nch0 = (v0 + C - 1) / C;
    if (v0 > 0 && min(N, nch0) <= S) {
      issue_item((int)blockIdx.x / H, (int)blockIdx.x % H, 0, v0, nch0);
      v0 = 0;  // issued
    }
  }

  // ---- 1. items per pair: their prefix over sequences, and that of the queued ones (all
  //      but the items CTAs started on) ----------------------------------------------------
  for (int i = tid; i < B; i += blockDim.x) {
    const int raw = p.valid_lens[i];
    if (raw > p.T_max) set_error(p.err, SPD_DEVERR_LENGTH);
    const int v = clamp_valid(raw, p.T_max);
    val_s[i] = v;
    nch_s[i] = (v + C - 1) / C;
    const int ib = (nch_s[i] + N - 1) / N;
    const int started = v > 0 ? min(max(G - i * H, 0), H) : 0;
    ip[i + 1] = ib * H;
    qp[i + 1] = ib * H - started;
  }
  if (tid == 0) {
    ip[0] = 0;
    qp[0] = 0;
  }
  __syncthreads();
  if (warp < 2) {
    int* pre = warp == 0 ? ip : qp;
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int i = base + lane;
      int v = (i < B) ? pre[i + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (i < B) pre[i + 1] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    if (val_s[b] == 0) {
      for (int i = tid; i < H * D; i += blockDim.x) out[(size_t)b * H * D + i] = Elem<T>::from_f(0.f);
    }
  }

  // ---- 2. producer warp: the queued items ------------------------------------------------
  if (warp == NW) {
    if (lane == 0) {
      if (v0 > 0) issue_item((int)blockIdx.x / H, (int)blockIdx.x % H, 0, v0, nch0);  // deferred first item
      const int n_queue = qp[B];
      int q = atomicAdd(next_item, 1);
      while (alive && q < n_queue) {
        const int nxt = atomicAdd(next_item, 1);  // next take, in flight meanwhile
        const int b = upper_index_i32(qp, B, q);
        const int ib = (nch_s[b] + N - 1) / N;  // items of each pair of sequence b
        const int hs = val_s[b] > 0 ? min(max(G - b * H, 0), H) : 0;  // pairs whose item 0 was started
        const int r = q - qp[b];
        int h, k;
        if (ib > 1 && r < hs * (ib - 1)) {
          h = r / (ib - 1);
          k = 1 + r % (ib - 1);
        } else {
          const int r2 = r - hs * (ib - 1);
          h = hs + r2 / ib;
          k = r2 % ib;
        }
        issue_item(b, h, k, val_s[b], nch_s[b]);
        q = nxt;
      }
      // end-of-work stage for the compute warps
      if (alive && n_issued >= S && !mbar_wait_bounded(&empty[s_p], ph_p ^ 1, p.err, p.wait_ns)) alive = false;
      if (alive) {
        meta[s_p] = CrossStage{-1, 0, 0, 0, 0, 0, 0, 0};
        mbar_arrive(&full[s_p]);
      } else {
        flag[0] = 1;
      }
      // this CTA takes no more items; the last CTA to get here re-arms the counter
      __threadfence();
      if (atomicAdd(done_ctas, 1) == G - 1) {
        *((volatile int*)next_item) = 0;
        *((volatile int*)done_ctas) = 0;
        __threadfence();
      }
      // after an abort, copies still in flight land before shared memory is released
      if (!alive) {
        for (int k = 0; k < S && k < n_issued; ++k) {
          const long long u = n_issued - 1 - k;
          (void)mbar_wait_bounded(&full[u % S], (uint32_t)((u / S) & 1), nullptr);
        }
      }
    }
    return;
  }

  // ---- 3. compute warps -----------------------------------------------------------------
  const int r = lane / LPR, sub = lane % LPR, rot = r % NCH;
  const int dl = lane % PVL, rg = lane / PVL;
  float qr[DPL];
  float m = -INFINITY, l = 0.f, acc[DPV];
  int s = 0;
  uint32_t ph = 0;

  for (;;) {
    if (*((volatile int*)&flag[0]) || !mbar_wait_bounded(&full[s], ph, p.err, p.wait_ns)) {
      flag[0] = 1;
      break;
    }
    const CrossStage mt = meta[s];
    if (mt.b < 0) break;
    const int b = mt.b, h = mt.h, j = mt.j;
    const int nrows = min(C, val_s[b] - j * C);
    const T* Ks = ring + (size_t)s * stage_elems;
    const T* Vs = Ks + unit_elems;
    if (mt.flags & kCrossFirst) {
      m = -INFINITY;
      l = 0.f;
#pragma unroll
      for (int i = 0; i < DPV; ++i) acc[i] = 0.f;
      const T* qrow = Vs + unit_elems + sub * DPL;  // q row arrived with this unit
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int ci = (cc + rot) % NCH;
#pragma unroll
        for (int e = 0; e < CH; ++e) qr[cc * CH + e] = Elem<T>::to_f(qrow[ci * CH + e]) * p.scale_log2;
      }
    }
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int row0 = (ps * NW + warp) * RPP;
      if (row0 >= nrows) break;  // warp-uniform
      const int nv = min(RPP, nrows - row0);
      float sc = -INFINITY;
      if (r < nv) {
        const T* krow = Ks + (size_t)(row0 + r) * D + sub * DPL;
        float dot = 0.f;
#pragma unroll
        for (int cc = 0; cc < NCH; ++cc) {
          const int ci = (cc + rot) % NCH;
          float kv[CH];
          load_to_float<T, CH>(krow + ci * CH, kv);
#pragma unroll
          for (int e = 0; e < CH; ++e) dot = fmaf(qr[cc * CH + e], kv[e], dot);
        }
        sc = dot;
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
      if (r >= nv) sc = -INFINITY;
      const float mnew = fmaxf(m, warp_max(sc));
      const float alpha = exp2f(m - mnew);
      const float pr = (r < nv) ? exp2f(sc - mnew) : 0.f;
      l = l * alpha + (sub == 0 ? pr : 0.f);
#pragma unroll
      for (int i = 0; i < DPV; ++i) acc[i] *= alpha;
      m = mnew;
      for (int r0 = 0; r0 < nv; r0 += PRG) {
        const int rr = r0 + rg;
        const float prr = __shfl_sync(0xffffffffu, pr, min(rr, RPP - 1) * LPR);
        if (rr < nv) {
          float vv[DPV];
          load_to_float<T, DPV>(Vs + (size_t)(row0 + rr) * D + dl * DPV, vv);
#pragma unroll
          for (int i = 0; i < DPV; ++i) acc[i] = fmaf(prr, vv[i], acc[i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }
    if (!(mt.flags & kCrossLast)) continue;

    // ---- item end: merge the compute warps' states in shared memory -----------------------
    const float lw = warp_sum(l);
    if constexpr (PRG > 1) {
#pragma unroll
      for (int o = PVL; o < 32; o <<= 1)
#pragma unroll
        for (int i = 0; i < DPV; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
    float* mw = merge + warp * (D + 2);
    if (rg == 0) {
#pragma unroll
      for (int i = 0; i < DPV; ++i) mw[dl * DPV + i] = acc[i];
    }
    if (lane == 0) {
      mw[D] = m;
      mw[D + 1] = lw;
    }
    named_sync(kCrossComputeBarrier, NCT);
    if (warp == 0) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, merge[w * (D + 2) + D]);
      float L = 0.f, o[DPV];
#pragma unroll
      for (int i = 0; i < DPV; ++i) o[i] = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float mwv = merge[w * (D + 2) + D];
        const float wt = (mwv == -INFINITY) ? 0.f : exp2f(mwv - M);
        L = fmaf(merge[w * (D + 2) + D + 1], wt, L);
#pragma unroll
        for (int i = 0; i < DPV; ++i) o[i] = fmaf(merge[w * (D + 2) + dl * DPV + i], wt, o[i]);
      }
      if ((nch_s[b] + N - 1) / N == 1) {  // the item is the whole pair
        if (rg == 0) {
          const float inv = 1.f / L;
          T* op = out + ((size_t)b * H + h) * D + dl * DPV;
#pragma unroll
          for (int i = 0; i < DPV; ++i) op[i] = Elem<T>::from_f(o[i] * inv);
        }
      } else {  // a partial for the merge kernel, kept in L2
        const int ib = (nch_s[b] + N - 1) / N;
        float* slot = p.partials + ((size_t)ip[b] + (size_t)h * ib + mt.item) * (D + 2);
        const uint64_t keep = l2_policy_evict_last();
        if (rg == 0) {
          if constexpr (DPV % 2 == 0) {
#pragma unroll
            for (int i = 0; i < DPV; i += 2) st_global_hint(slot + dl * DPV + i, make_float2(o[i], o[i + 1]), keep);
          } else {
#pragma unroll
            for (int i = 0; i < DPV; ++i) slot[dl * DPV + i] = o[i];
          }
        }
        if (lane == 0) st_global_hint(slot + D, make_float2(M, L), keep);
      }
    }
    named_sync(kCrossComputeBarrier, NCT);  // the merge buffer is reused by the next item
  }
}

// ------------------------------------------------------------------ merge kernel
// One warp per (b, h) pair that spans more than one item; launched with programmatic
// dependent launch behind the streaming kernel.  The pair's first item index (the sum of
// the items of the sequences before b, plus h times b's items per pair) is worked out from
// the valid lengths while the streaming kernel still runs: it never writes them and
// triggers this launch at its start, before which everything it reads is final.  After
// griddepcontrol.wait every partial of the pair is loaded in one round of loads.
template <typename T, int D, int C>
__global__ void __launch_bounds__(128) cross_merge_kernel(const CrossParams p) {
  constexpr int EPL = D >= 64 ? D / 32 : 2;  // acc elements per lane
  using V = std::conditional_t<EPL == 4, float4, float2>;
  static_assert(EPL == 2 || EPL == 4, "head_dim");
  const int lane = threadIdx.x & 31;
  const long long pair = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const bool live = pair < (long long)p.B * p.H;
  const int b = live ? (int)(pair / p.H) : 0, h = live ? (int)(pair % p.H) : 0;
  const int N = p.item_units;
  auto items_of = [&](int bb) { return ((clamp_valid(p.valid_lens[bb], p.T_max) + C - 1) / C + N - 1) / N; };
  const int nitems = live ? items_of(b) : 0;
  int i0 = 0;
  for (int bb = lane; bb < b && live; bb += 32) i0 += items_of(bb);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) i0 += __shfl_xor_sync(0xffffffffu, i0, o);
  i0 = i0 * p.H + h * nitems;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the streaming kernel has finished
  if (!live || nitems <= 1) return;                    // written by the streaming kernel (or zero)
  const float* base = p.partials + (size_t)i0 * (D + 2);
  float2 ml = make_float2(-INFINITY, 0.f);
  if (lane < nitems) ml = __ldcg(reinterpret_cast<const float2*>(base + (size_t)lane * (D + 2) + D));
  const bool hold = lane < D / EPL;
  V a[kCrossMaxItems];
#pragma unroll
  for (int it = 0; it < kCrossMaxItems; ++it) {
    a[it] = V{};
    if (it < nitems && hold) {  // rows of D + 2 floats: 8-byte aligned, so two-float loads
      const float2* src = reinterpret_cast<const float2*>(base + (size_t)it * (D + 2) + lane * EPL);
      const float2 x0 = __ldcg(src);
      a[it].x = x0.x;
      a[it].y = x0.y;
      if constexpr (EPL == 4) {
        const float2 x1 = __ldcg(src + 1);
        a[it].z = x1.x;
        a[it].w = x1.y;
      }
    }
  }
  const float M = warp_max(ml.x);
  const float w = lane < nitems ? exp2f(ml.x - M) : 0.f;
  const float inv = 1.f / warp_sum(ml.y * w);
  V o{};
#pragma unroll
  for (int it = 0; it < kCrossMaxItems; ++it) {
    const float wi = __shfl_sync(0xffffffffu, w, it);
    o.x = fmaf(wi, a[it].x, o.x);
    o.y = fmaf(wi, a[it].y, o.y);
    if constexpr (EPL == 4) {
      o.z = fmaf(wi, a[it].z, o.z);
      o.w = fmaf(wi, a[it].w, o.w);
    }
  }
  if (hold) {
    T* dst = reinterpret_cast<T*>(p.out) + ((size_t)b * p.H + h) * D + lane * EPL;
    dst[0] = Elem<T>::from_f(o.x * inv);
    dst[1] = Elem<T>::from_f(o.y * inv);
    if constexpr (EPL == 4) {
      dst[2] = Elem<T>::from_f(o.z * inv);
      dst[3] = Elem<T>::from_f(o.w * inv);
    }
  }
}

template <typename T, int D>
static int launch_cross(const CrossParams& base, int sms, cudaStream_t stream) {
  using Gm = CrossGeom<T, D>;
  CrossParams p = base;
  // items of 2+ units, at most kCrossMaxItems per pair
  const int nch_max = (p.T_max + Gm::C - 1) / Gm::C;
  const int n_by_cap = (nch_max + kCrossMaxItems - 1) / kCrossMaxItems;
  p.item_units = n_by_cap > 2 ? n_by_cap : 2;
  const size_t stage_bytes = ((size_t)2 * Gm::C + 1) * D * sizeof(T);
  // ~96 KB of stages per CTA: two CTAs per SM, each with a producer warp streaming.
  int S = (int)((96 * 1024) / stage_bytes);
  S = S < 2 ? 2 : (S > 8 ? 8 : S);
  p.stages = S;
  const size_t smem = round_up((size_t)S * stage_bytes, 128) + 16 * (size_t)S + sizeof(CrossStage) * (size_t)S +
                      4 * (size_t)Gm::NW * (D + 2) + 4 * (4 * (size_t)p.B + 6);
  if (smem > 227 * 1024) return SPD_ERR_UNSUPPORTED;
  auto kfn = cross_attn_kernel<T, D>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SPD_ERR_CUDA;
  int occ = 0;
  const int threads = (Gm::NW + 1) * 32;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, threads, smem) != cudaSuccess || occ < 1)
    return SPD_ERR_CUDA;
  if (occ > kMaxCtasPerSm) occ = kMaxCtasPerSm;
  kfn<<<sms * occ, threads, smem, stream>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return SPD_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((long long)p.B * p.H + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cross_merge_kernel<T, D, Gm::C>, p) == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

template <typename T>
static int cross_dispatch_d(const CrossParams& p, int D, int sms, cudaStream_t st) {
  switch (D) {
    case 16: return launch_cross<T, 16>(p, sms, st);
    case 32: return launch_cross<T, 32>(p, sms, st);
    case 64: return launch_cross<T, 64>(p, sms, st);
    case 128: return launch_cross<T, 128>(p, sms, st);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

int cross_attn_launch(const CrossParams& p, int dtype, int D, int sms, cudaStream_t st) {
  switch (dtype) {
    case SPD_F32: return cross_dispatch_d<float>(p, D, sms, st);
    case SPD_F16: return cross_dispatch_d<__half>(p, D, sms, st);
    case SPD_BF16: return cross_dispatch_d<__nv_bfloat16>(p, D, sms, st);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

}  // namespace spd
