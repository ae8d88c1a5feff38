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
// * Work units are pool blocks.  A unit covers one block of ALL heads, which in the
//   pool layout [num_blocks][block_size][H][D] is one contiguous run of
//   block_size*H*D elements, fetched with two 1-D bulk async copies (K and V; only the
//   valid rows of a sequence's last block).
// * Units of all sequences are laid end to end and every CTA of a persistent grid
//   (num_SMs x resident CTAs) streams an equal contiguous share, so load balance does
//   not depend on the context-length distribution.
// * Warp specialisation: one producer warp (lane 0) runs ahead through an S-stage
//   shared-memory ring (full mbarriers complete on the copies' bytes; empty mbarriers
//   collect one arrival per compute warp), so compute warps never meet a CTA-wide
//   barrier per unit.  Compute warp w owns heads [w*HPW, (w+1)*HPW).
// * q·k: 32/block_size lanes per row, q (pre-scaled by scale*log2 e) in registers, K
//   chunks read in a per-row rotated order so the 8 lanes of a shared-memory phase hit
//   distinct banks.  p·v: each lane owns one 16-byte chunk of a row and the warp walks
//   32/chunks_per_row rows at a time; partial sums across row groups are folded once per
//   sequence.  Online softmax in base 2; packed fp32x2 FMAs throughout.
// * A sequence split across CTAs is merged by the last CTA to finish it: each CTA writes
//   (m, l, acc) per head to partial slot (b + c); after a CTA barrier one thread fences
//   and bumps the sequence's arrival counter; the last arrival combines the partials
//   and resets the counter (no spinning, no second launch).
#include "spd_params.cuh"

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

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
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

constexpr int kPagedComputeBarrier = 1;  // named barrier among compute warps
constexpr int kIdsWindow = 256;          // block ids preloaded per CTA

template <typename T, int D, int BS, int HPW>
__global__ void __launch_bounds__(544) paged_decode_attn_kernel(const PagedParams p) {
  using Gm = PagedGeom<T, D, BS>;
  constexpr int LPR = Gm::LPR, DPL = Gm::DPL, CH = Gm::CH, NCH = Gm::NCH;
  constexpr int VE = Gm::VE, CPR = Gm::CPR, RG = Gm::RG, PVP = Gm::PVP;

  extern __shared__ __align__(128) unsigned char smem[];
  const int H = p.H, B = p.B, S = p.stages;
  const int HD = H * D;
  const int NW = (H + HPW - 1) / HPW;  // compute warps; warp NW is the producer
  const int NCT = NW * 32;             // compute threads
  const size_t unit_elems = (size_t)BS * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Stage s: K block, V block, then q / k_new / v_new rows of the unit's sequence.
  const size_t stage_elems = 2 * unit_elems + 3 * (size_t)HD;
  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + round_up((size_t)S * stage_elems * sizeof(T), 128));
  uint64_t* empty = full + S;
  int* prefix = reinterpret_cast<int*>(empty + S);  // [B + 1] unit prefix over sequences
  int* ctx_s = prefix + B + 1;                      // [B] clamped context lengths
  int* flag = ctx_s + B;                            // [0] last-arrival, [1] abort
  int* ids = flag + 2;                              // [kIdsWindow] block ids of this CTA's units

  const T* __restrict__ kpool = reinterpret_cast<const T*>(p.k_pool);
  const T* __restrict__ vpool = reinterpret_cast<const T*>(p.v_pool);
  T* __restrict__ out = reinterpret_cast<T*>(p.out);
  const T* __restrict__ qg = reinterpret_cast<const T*>(p.q);
  const bool append = p.k_new != nullptr;
  const int max_ctx = p.max_blocks * BS;

  // ---- 1. unit prefix over sequences (every CTA computes it; B is small) ----------
  for (int i = tid; i < B; i += blockDim.x) {
    int c = p.context_lens[i];
    if (c > max_ctx) {
      set_error(p.err, SPD_DEVERR_LENGTH);
      c = max_ctx;
    }
    c = c > 0 ? c : 0;
    ctx_s[i] = c;
    prefix[i + 1] = (c + BS - 1) / BS;
  }
  if (tid == 0) {
    prefix[0] = 0;
    flag[1] = 0;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int i = base + lane;
      int v = (i < B) ? prefix[i + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (i < B) prefix[i + 1] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();

  const long long W = prefix[B];
  // Effective grid: never more CTAs than units, so every participating CTA owns at
  // least one unit and the CTAs sharing a sequence are consecutive (which the arrival
  // count nparts = c_last - c_first + 1 relies on).
  const int c = blockIdx.x;
  const int G = (int)((long long)gridDim.x < W ? (long long)gridDim.x : W);

  // ---- 2. sequences with nothing to attend to get zeros (CTA b % gridDim) ----------
  for (int b = c; b < B; b += gridDim.x) {
    if (prefix[b + 1] == prefix[b]) {
      for (int i = tid; i < HD; i += blockDim.x) out[(size_t)b * HD + i] = Elem<T>::from_f(0.f);
    }
  }
  if (W == 0 || c >= G) return;
  const long long start = range_start(c, G, W), end = range_start(c + 1, G, W);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_barrier_init();
  }
  // Block ids of the first kIdsWindow units of this CTA, loaded in parallel (one round
  // trip) so the producer never waits on a block-table load.
  {
    const long long nids = min(end - start, (long long)kIdsWindow);
    for (long long i = tid; i < nids; i += blockDim.x) {
      const long long u = start + i;
      const int bb = upper_index_i32(prefix, B, u);
      int phys = p.block_tables[(size_t)bb * p.max_blocks + (u - prefix[bb])];
      if (phys < 0 || phys >= p.num_blocks) {
        set_error(p.err, SPD_DEVERR_BLOCK_ID);
        phys = 0;
      }
      ids[i] = phys;
    }
  }
  __syncthreads();

  // ---- 3. producer warp -------------------------------------------------------------
  if (warp == NW) {
    if (lane == 0) {
      int pb = upper_index_i32(prefix, B, start);
      int s = 0;
      uint32_t ph = 0;
      long long issued = start;
      for (long long u = start; u < end; ++u) {
        if (u - start >= S) {
          if (*((volatile int*)&flag[1]) || !mbar_wait_bounded(&empty[s], ph ^ 1, p.err)) {
            flag[1] = 1;
            break;
          }
        }
        while (prefix[pb + 1] <= u) ++pb;
        const int j = (int)(u - prefix[pb]);
        const int nvalid = min(BS, ctx_s[pb] - j * BS);
        int phys;
        if (u - start < kIdsWindow) {
          phys = ids[u - start];
        } else {
          phys = p.block_tables[(size_t)pb * p.max_blocks + j];
          if (phys < 0 || phys >= p.num_blocks) {
            set_error(p.err, SPD_DEVERR_BLOCK_ID);
            phys = 0;
          }
        }
        const size_t off = (size_t)phys * unit_elems;
        const uint32_t bytes = (uint32_t)(nvalid * HD * (int)sizeof(T));
        const uint32_t row_bytes = (uint32_t)(HD * (int)sizeof(T));
        const bool seg_first = (u == start) || (u == prefix[pb]);
        const bool app = append && (j == prefix[pb + 1] - prefix[pb] - 1);
        T* dst = ring + (size_t)s * stage_elems;
        mbar_arrive_expect_tx(&full[s], 2 * bytes + (seg_first ? row_bytes : 0u) + (app ? 2 * row_bytes : 0u));
        bulk_copy_g2s(dst, kpool + off, bytes, &full[s]);
        bulk_copy_g2s(dst + unit_elems, vpool + off, bytes, &full[s]);
        if (seg_first) bulk_copy_g2s(dst + 2 * unit_elems, qg + (size_t)pb * HD, row_bytes, &full[s]);
        if (app) {
          bulk_copy_g2s(dst + 2 * unit_elems + HD, reinterpret_cast<const T*>(p.k_new) + (size_t)pb * HD, row_bytes,
                        &full[s]);
          bulk_copy_g2s(dst + 2 * unit_elems + 2 * HD, reinterpret_cast<const T*>(p.v_new) + (size_t)pb * HD,
                        row_bytes, &full[s]);
        }
        issued = u + 1;
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      // Copies still in flight land before this CTA's shared memory is released:
      // wait (bounded) for the last phase of every stage that was used.
      const long long n = issued - start;
      for (int k = 0; k < S && k < n; ++k) {
        const long long u = issued - 1 - k;
        const int st = (int)((u - start) % S);
        (void)mbar_wait_bounded(&full[st], (uint32_t)(((u - start) / S) & 1), nullptr);
      }
    }
    return;
  }

  // ---- 4. compute warps -----------------------------------------------------------------
  const int r = lane / LPR;    // q·k row of this lane
  const int sub = lane % LPR;  // which DPL-slice of the row
  const int rot = r & (NCH - 1);
  const int cidx = lane % CPR;  // p·v chunk of this lane
  const int rg = lane / CPR;    // p·v row group

  float2 qr[HPW][DPL / 2];
  float m[HPW], l[HPW];
  float2 acc[HPW][VE / 2];

  int b = upper_index_i32(prefix, B, start);
  bool need_q = true;
  int s = 0;
  uint32_t ph = 0;

  for (long long g = start; g < end; ++g) {
    const bool ok = !*((volatile int*)&flag[1]) && mbar_wait_bounded(&full[s], ph, p.err);
    if (!ok) flag[1] = 1;
    const int j = (int)(g - prefix[b]);
    const int nblk = prefix[b + 1] - prefix[b];
    const int nvalid = min(BS, ctx_s[b] - j * BS);
    T* Ks = ring + (size_t)s * stage_elems;
    T* Vs = Ks + unit_elems;
    const T* Qs = Vs + unit_elems;  // q row of sequence b (first unit of a segment only)

    if (need_q) {
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        m[k] = -INFINITY;
        l[k] = 0.f;
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) acc[k][i] = make_float2(0.f, 0.f);
        if (h < H && ok) {
          const T* qrow = Qs + h * D + sub * DPL;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            const int ci = (cc + rot) & (NCH - 1);
            load_f2<T, CH>(qrow + ci * CH, &qr[k][cc * CH / 2]);
#pragma unroll
            for (int e = 0; e < CH / 2; ++e) {
              qr[k][cc * CH / 2 + e].x *= p.scale_log2;
              qr[k][cc * CH / 2 + e].y *= p.scale_log2;
            }
          }
        }
      }
      need_q = false;
    }

    if (append && j == nblk - 1) {
      // op (3) fused: the new token sits at row nvalid-1 of the sequence's last block.
      int phys = p.block_tables[(size_t)b * p.max_blocks + j];
      if (phys < 0 || phys >= p.num_blocks) phys = 0;  // flagged by the producer
      const size_t row_off = (size_t)(nvalid - 1) * HD;
      T* kdst = const_cast<T*>(kpool) + (size_t)phys * unit_elems + row_off;
      T* vdst = const_cast<T*>(vpool) + (size_t)phys * unit_elems + row_off;
      const T* ksrc = Qs + HD;  // k_new / v_new rows arrived with this unit
      const T* vsrc = Qs + 2 * HD;
      constexpr int VEC = 16 / sizeof(T);
      if (ok) {
        for (int i = tid * VEC; i < HD; i += NCT * VEC) {
          const uint4 kv = *reinterpret_cast<const uint4*>(ksrc + i);
          const uint4 vv = *reinterpret_cast<const uint4*>(vsrc + i);
          *reinterpret_cast<uint4*>(Ks + row_off + i) = kv;
          *reinterpret_cast<uint4*>(Vs + row_off + i) = vv;
          *reinterpret_cast<uint4*>(kdst + i) = kv;
          *reinterpret_cast<uint4*>(vdst + i) = vv;
        }
      }
      fence_proxy_async_smem();  // generic writes before the next bulk copy into this stage
      named_sync(kPagedComputeBarrier, NCT);
    }

    if (ok) {
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        if (h >= H) continue;
        const T* Kh = Ks + h * D;
        const T* Vh = Vs + h * D;
        // q·k for row r
        float sc = -INFINITY;
        if (r < nvalid) {
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
        if (r >= nvalid) sc = -INFINITY;
        const float mnew = fmaxf(m[k], warp_max(sc));
        const float alpha = exp2f(m[k] - mnew);
        const float pr = (r < nvalid) ? exp2f(sc - mnew) : 0.f;
        l[k] = l[k] * alpha + (sub == 0 ? pr : 0.f);
        m[k] = mnew;
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int i = 0; i < VE / 2; ++i) acc[k][i] = __fmul2_rn(acc[k][i], a2);
        // p·v: this lane's 16-byte chunk of rows rg, rg+RG, ...
#pragma unroll
        for (int ps = 0; ps < PVP; ++ps) {
          const int rr = ps * RG + rg;
          const float prr = __shfl_sync(0xffffffffu, pr, (rr < BS ? rr : 0) * LPR);
          if (rr < nvalid) {
            float2 vv[VE / 2];
            load_f2<T, VE>(Vh + (size_t)rr * HD + cidx * VE, vv);
            const float2 p2 = make_float2(prr, prr);
#pragma unroll
            for (int i = 0; i < VE / 2; ++i) acc[k][i] = __ffma2_rn(p2, vv[i], acc[k][i]);
          }
        }
      }
    }
    // this warp is done with stage s
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }

    // ---- segment end: finish sequence b -------------------------------------------
    const bool seq_end = (g + 1 == prefix[b + 1]);
    if (seq_end || g + 1 == end) {
      const bool whole = (start <= prefix[b]) && (end >= prefix[b + 1]);
      float ltot[HPW];
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        ltot[k] = warp_sum(l[k]);
#pragma unroll
        for (int o = CPR; o < 32; o <<= 1)
#pragma unroll
          for (int i = 0; i < VE / 2; ++i) {
            acc[k][i].x += __shfl_xor_sync(0xffffffffu, acc[k][i].x, o);
            acc[k][i].y += __shfl_xor_sync(0xffffffffu, acc[k][i].y, o);
          }
      }
      if (whole) {
#pragma unroll
        for (int k = 0; k < HPW; ++k) {
          const int h = warp * HPW + k;
          if (h < H && rg == 0) {
            const float inv = 1.f / ltot[k];
            T* o = out + ((size_t)b * H + h) * D + cidx * VE;
#pragma unroll
            for (int i = 0; i < VE / 2; ++i) {
              o[2 * i] = Elem<T>::from_f(acc[k][i].x * inv);
              o[2 * i + 1] = Elem<T>::from_f(acc[k][i].y * inv);
            }
          }
        }
      } else {
        const long long p0 = prefix[b], p1 = prefix[b + 1];
        const int c_first = cta_of_unit(p0, G, W);
        const int c_last = cta_of_unit(p1 - 1, G, W);
        const int nparts = c_last - c_first + 1;
#pragma unroll
        for (int k = 0; k < HPW; ++k) {
          const int h = warp * HPW + k;
          if (h < H) {
            float* slot = p.partials + ((size_t)(b + c) * H + h) * (D + 2);
            if (rg == 0) {
#pragma unroll
              for (int i = 0; i < VE / 2; ++i)
                *reinterpret_cast<float2*>(slot + cidx * VE + 2 * i) = acc[k][i];
            }
            if (lane == 0) {
              slot[D] = m[k];
              slot[D + 1] = ltot[k];
            }
          }
        }
        // every compute thread's partial writes precede thread 0's fence + arrival
        named_sync(kPagedComputeBarrier, NCT);
        if (tid == 0) {
          __threadfence();
          const int old = atomicAdd(&p.counters[b], 1);
          const int last = (old == nparts - 1);
          if (last) {
            p.counters[b] = 0;  // every part has arrived; ready for the next call
            __threadfence();
          }
          flag[0] = last;
        }
        named_sync(kPagedComputeBarrier, NCT);
        if (flag[0]) {
          for (int h = warp; h < H; h += NW) {
            float M = -INFINITY;
            for (int cc = c_first; cc <= c_last; ++cc)
              M = fmaxf(M, __ldcg(p.partials + ((size_t)(b + cc) * H + h) * (D + 2) + D));
            float L = 0.f;
            float2 o[VE / 2];
#pragma unroll
            for (int i = 0; i < VE / 2; ++i) o[i] = make_float2(0.f, 0.f);
            for (int cc = c_first; cc <= c_last; ++cc) {
              const float* slot = p.partials + ((size_t)(b + cc) * H + h) * (D + 2);
              const float w = exp2f(__ldcg(slot + D) - M);
              L = fmaf(__ldcg(slot + D + 1), w, L);
              const float2 w2 = make_float2(w, w);
#pragma unroll
              for (int i = 0; i < VE / 2; ++i)
                o[i] = __ffma2_rn(__ldcg(reinterpret_cast<const float2*>(slot + cidx * VE + 2 * i)), w2, o[i]);
            }
            if (rg == 0) {
              const float inv = 1.f / L;
              T* op = out + ((size_t)b * H + h) * D + cidx * VE;
#pragma unroll
              for (int i = 0; i < VE / 2; ++i) {
                op[2 * i] = Elem<T>::from_f(o[i].x * inv);
                op[2 * i + 1] = Elem<T>::from_f(o[i].y * inv);
              }
            }
          }
        }
      }
      if (seq_end) {
        ++b;
        while (b < B && prefix[b + 1] == prefix[b]) ++b;
        need_q = true;
      }
    }
  }
}

// ------------------------------------------------------------------ host launcher
template <typename T, int D, int BS, int HPW>
static int launch_paged(const PagedParams& base, int device_sms, cudaStream_t stream) {
  PagedParams p = base;
  const int nw = (p.H + HPW - 1) / HPW;
  const int threads = (nw + 1) * 32;
  const size_t stage_bytes = ((size_t)2 * BS + 3) * p.H * D * sizeof(T);
  // Ring depth: up to ~216 KB of stages per CTA (one CTA per SM at the Whisper shapes;
  // the producer warp keeps every stage in flight), at least two stages.
  const size_t fixed = 16 * 8 + 4 * (2 * (size_t)p.B + 3 + kIdsWindow) + 256;
  int S = (int)((216 * 1024 - fixed) / stage_bytes);
  if (S < 2 && 2 * stage_bytes + fixed <= 227 * 1024) S = 2;
  S = S < 1 ? 1 : (S > 8 ? 8 : S);
  p.stages = S;
  const size_t smem = round_up((size_t)S * stage_bytes, 128) + 16 * (size_t)S +
                      4 * (2 * (size_t)p.B + 3 + kIdsWindow);
  if (smem > 227 * 1024) return SPD_ERR_UNSUPPORTED;
  auto kfn = paged_decode_attn_kernel<T, D, BS, HPW>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SPD_ERR_CUDA;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, threads, smem) != cudaSuccess || occ < 1)
    return SPD_ERR_CUDA;
  if (occ > kMaxCtasPerSm) occ = kMaxCtasPerSm;
  kfn<<<device_sms * occ, threads, smem, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

template <typename T, int D>
static int dispatch_bs(const PagedParams& p, int bs, int sms, cudaStream_t st) {
  const bool two = p.H > 16;
  switch (bs) {
    case 8: return two ? launch_paged<T, D, 8, 2>(p, sms, st) : launch_paged<T, D, 8, 1>(p, sms, st);
    case 16: return two ? launch_paged<T, D, 16, 2>(p, sms, st) : launch_paged<T, D, 16, 1>(p, sms, st);
    case 32:
      if constexpr (D <= 64) {
        return two ? launch_paged<T, D, 32, 2>(p, sms, st) : launch_paged<T, D, 32, 1>(p, sms, st);
      }
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
