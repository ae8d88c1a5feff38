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
//   block_size*H*D elements, so each unit is fetched with two 1-D bulk async copies
//   (K and V; only the valid rows of a sequence's last block are copied).
// * Units of all sequences are laid end to end and every CTA of a persistent grid
//   (num_SMs x resident CTAs) streams an equal contiguous share through an S-stage
//   shared-memory ring whose stages complete on mbarriers.  Load balance is therefore
//   independent of the context-length distribution.
// * A sequence split across CTAs is merged by the last CTA to finish it (arrival
//   counter + fences, no spinning): each CTA writes (m, l, acc) per head to a partial
//   slot indexed (b + c); the last arrival combines them and resets the counter.
// * Warp w owns heads [w*HPW, (w+1)*HPW).  Q·K: LPR = 32/block_size lanes per row,
//   each lane keeping its share of q (pre-scaled by scale*log2 e) in registers, read in
//   a per-row rotated chunk order so the 8 lanes of a shared-memory phase hit distinct
//   banks.  Online softmax in base 2 with warp shuffles.  P·V: each lane owns D/32 dims.
#include "spd_params.cuh"

namespace spd {

template <typename T, int D, int BS>
struct PagedGeom {
  static constexpr int EB = sizeof(T);
  static constexpr int LPR = 32 / BS;                        // lanes per row for q·k
  static constexpr int DPL = D / LPR;                        // dims per lane for q·k
  static constexpr int CH = (DPL * EB >= 16) ? 16 / EB : DPL;  // elems per smem chunk
  static constexpr int NCH = DPL / CH;                       // chunks per lane
  static constexpr int PVL = D >= 32 ? 32 : D;               // lanes per row for p·v
  static constexpr int PRG = 32 / PVL;                       // row groups for p·v
  static constexpr int DPV = D / PVL;                        // dims per lane for p·v
  static_assert(LPR >= 1 && LPR * BS == 32, "block_size must divide 32");
  static_assert(DPL * LPR == D && DPV * PVL == D, "bad head_dim");
};

template <typename T, int D, int BS, int HPW>
__global__ void __launch_bounds__(512) paged_decode_attn_kernel(const PagedParams p) {
  using Gm = PagedGeom<T, D, BS>;
  constexpr int LPR = Gm::LPR, DPL = Gm::DPL, CH = Gm::CH, NCH = Gm::NCH;
  constexpr int PVL = Gm::PVL, PRG = Gm::PRG, DPV = Gm::DPV;

  extern __shared__ __align__(128) unsigned char smem[];
  const int H = p.H, B = p.B, S = p.stages;
  const int HD = H * D;
  const size_t unit_elems = (size_t)BS * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;

  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + round_up((size_t)S * 2 * unit_elems * sizeof(T), 128));
  int* prefix = reinterpret_cast<int*>(bars + S);  // [B + 1] unit prefix over sequences
  int* ctx_s = prefix + B + 1;                     // [B] clamped context lengths
  int* flag = ctx_s + B;                           // [1] "this CTA finishes the sequence"

  const T* __restrict__ kpool = reinterpret_cast<const T*>(p.k_pool);
  const T* __restrict__ vpool = reinterpret_cast<const T*>(p.v_pool);
  T* __restrict__ out = reinterpret_cast<T*>(p.out);
  const T* __restrict__ qg = reinterpret_cast<const T*>(p.q);
  const bool append = p.k_new != nullptr;
  const int max_ctx = p.max_blocks * BS;

  // ---- 1. unit prefix over sequences (every CTA computes it; B is small) ----------
  for (int i = tid; i < B; i += nthreads) {
    int c = p.context_lens[i];
    if (c > max_ctx) {
      set_error(p.err, SPD_DEVERR_LENGTH);
      c = max_ctx;
    }
    c = c > 0 ? c : 0;
    ctx_s[i] = c;
    prefix[i + 1] = (c + BS - 1) / BS;
  }
  if (tid == 0) prefix[0] = 0;
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
  // least one unit and the CTAs sharing a segment are consecutive (which the
  // arrival count nparts = c_last - c_first + 1 relies on).
  const int c = blockIdx.x;
  const int G = (int)((long long)gridDim.x < W ? (long long)gridDim.x : W);

  // ---- 2. sequences with nothing to attend to get zeros (CTA b % G) ---------------
  for (int b = c; b < B; b += gridDim.x) {
    if (prefix[b + 1] == prefix[b]) {
      for (int i = tid; i < HD; i += nthreads) out[(size_t)b * HD + i] = Elem<T>::from_f(0.f);
    }
  }
  if (W == 0 || c >= G) return;
  const long long start = range_start(c, G, W), end = range_start(c + 1, G, W);
  if (start >= end) return;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  // ---- 3. producer (thread 0): issue unit u into stage (u - start) % S -------------
  int pb = upper_index_i32(prefix, B, start);
  long long issued = start;
  auto issue = [&](long long u) {
    while (prefix[pb + 1] <= u) ++pb;
    const int j = (int)(u - prefix[pb]);
    const int nvalid = min(BS, ctx_s[pb] - j * BS);
    int phys = p.block_tables[(size_t)pb * p.max_blocks + j];
    if (phys < 0 || phys >= p.num_blocks) {
      set_error(p.err, SPD_DEVERR_BLOCK_ID);
      phys = 0;
    }
    const size_t off = (size_t)phys * unit_elems;
    const uint32_t bytes = (uint32_t)(nvalid * HD * (int)sizeof(T));
    const int s = (int)((u - start) % S);
    T* dst = ring + (size_t)s * 2 * unit_elems;
    mbar_arrive_expect_tx(&bars[s], 2 * bytes);
    bulk_copy_g2s(dst, kpool + off, bytes, &bars[s]);
    bulk_copy_g2s(dst + unit_elems, vpool + off, bytes, &bars[s]);
  };
  if (tid == 0) {
    for (int k = 0; k < S && issued < end; ++k) issue(issued++);
  }

  // ---- 4. consumers ----------------------------------------------------------------
  const int r = lane / LPR;    // row of this lane for q·k
  const int sub = lane % LPR;  // which DPL-slice of the row
  const int rot = r % NCH;     // rotated chunk order (bank spreading)
  const int dl = lane % PVL;   // p·v: dims [dl*DPV, dl*DPV + DPV)
  const int rg = lane / PVL;   // p·v: row group

  float qr[HPW][DPL];
  float m[HPW], l[HPW], acc[HPW][DPV];

  int b = upper_index_i32(prefix, B, start);
  bool need_q = true;
  bool timed_out = false;
  long long abort_at = -1;  // first unit not consumed when a wait ran out

  for (long long g = start; g < end; ++g) {
    const int s = (int)((g - start) % S);
    const uint32_t parity = (uint32_t)(((g - start) / S) & 1);
    if (need_q) {
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        m[k] = -INFINITY;
        l[k] = 0.f;
#pragma unroll
        for (int i = 0; i < DPV; ++i) acc[k][i] = 0.f;
        if (h < H) {
          const T* qrow = qg + ((size_t)b * H + h) * D + sub * DPL;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            const int ci = (cc + rot) % NCH;
#pragma unroll
            for (int e = 0; e < CH; ++e) qr[k][cc * CH + e] = Elem<T>::to_f(qrow[ci * CH + e]) * p.scale_log2;
          }
        }
      }
      need_q = false;
    }

    const bool ok = mbar_wait_bounded(&bars[s], parity, p.err);
    const int j = (int)(g - prefix[b]);
    const int nblk = prefix[b + 1] - prefix[b];
    const int nvalid = min(BS, ctx_s[b] - j * BS);
    T* Ks = ring + (size_t)s * 2 * unit_elems;
    T* Vs = Ks + unit_elems;

    if (append && j == nblk - 1) {
      // op (3) fused: the new token sits at row nvalid-1 of the sequence's last block.
      int phys = p.block_tables[(size_t)b * p.max_blocks + j];
      if (phys < 0 || phys >= p.num_blocks) phys = 0;  // flagged by the producer
      const size_t row_off = (size_t)(nvalid - 1) * HD;
      T* kdst = const_cast<T*>(kpool) + (size_t)phys * unit_elems + row_off;
      T* vdst = const_cast<T*>(vpool) + (size_t)phys * unit_elems + row_off;
      const T* ksrc = reinterpret_cast<const T*>(p.k_new) + (size_t)b * HD;
      const T* vsrc = reinterpret_cast<const T*>(p.v_new) + (size_t)b * HD;
      constexpr int VEC = 16 / sizeof(T);
      if (ok) {
        for (int i = tid * VEC; i < HD; i += nthreads * VEC) {
          const uint4 kv = *reinterpret_cast<const uint4*>(ksrc + i);
          const uint4 vv = *reinterpret_cast<const uint4*>(vsrc + i);
          *reinterpret_cast<uint4*>(Ks + row_off + i) = kv;
          *reinterpret_cast<uint4*>(Vs + row_off + i) = vv;
          *reinterpret_cast<uint4*>(kdst + i) = kv;
          *reinterpret_cast<uint4*>(vdst + i) = vv;
        }
      }
      fence_proxy_async_smem();
      __syncthreads();
    }

    if (ok) {
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        const int h = warp * HPW + k;
        if (h >= H) continue;
        const T* Kh = Ks + h * D;
        const T* Vh = Vs + h * D;
        // q·k for row r (LPR lanes per row)
        float sc = -INFINITY;
        if (r < nvalid) {
          const T* krow = Kh + (size_t)r * HD + sub * DPL;
          float dot = 0.f;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            const int ci = (cc + rot) % NCH;
            float kv[CH];
            load_to_float<T, CH>(krow + ci * CH, kv);
#pragma unroll
            for (int e = 0; e < CH; ++e) dot = fmaf(qr[k][cc * CH + e], kv[e], dot);
          }
          sc = dot;
        }
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        if (r >= nvalid) sc = -INFINITY;
        const float mblk = warp_max(sc);
        const float mnew = fmaxf(m[k], mblk);
        const float alpha = exp2f(m[k] - mnew);
        const float pr = (r < nvalid) ? exp2f(sc - mnew) : 0.f;
        l[k] = l[k] * alpha + (sub == 0 ? pr : 0.f);
#pragma unroll
        for (int i = 0; i < DPV; ++i) acc[k][i] *= alpha;
        m[k] = mnew;
        // p·v: row groups of PVL lanes walk the valid rows
        for (int r0 = 0; r0 < nvalid; r0 += PRG) {
          const int rr = r0 + rg;
          const float prr = __shfl_sync(0xffffffffu, pr, min(rr, BS - 1) * LPR);
          if (rr < nvalid) {
            float vv[DPV];
            load_to_float<T, DPV>(Vh + (size_t)rr * HD + dl * DPV, vv);
#pragma unroll
            for (int i = 0; i < DPV; ++i) acc[k][i] = fmaf(prr, vv[i], acc[k][i]);
          }
        }
      }
    } else {
      timed_out = true;
    }

    // All warps are done with stage s: refill it.  The OR makes the abort decision
    // uniform across the CTA.
    if (__syncthreads_or(timed_out)) {
      abort_at = g;
      break;
    }
    if (tid == 0 && issued < end) issue(issued++);

    // ---- segment end: finish sequence b -------------------------------------------
    const bool seq_end = (g + 1 == prefix[b + 1]);
    if (seq_end || g + 1 == end) {
      const bool whole = (start <= prefix[b]) && (end >= prefix[b + 1]);
      float ltot[HPW];
#pragma unroll
      for (int k = 0; k < HPW; ++k) {
        ltot[k] = warp_sum(l[k]);
        if constexpr (PRG > 1) {
#pragma unroll
          for (int o = PVL; o < 32; o <<= 1)
#pragma unroll
            for (int i = 0; i < DPV; ++i) acc[k][i] += __shfl_xor_sync(0xffffffffu, acc[k][i], o);
        }
      }
      if (whole) {
#pragma unroll
        for (int k = 0; k < HPW; ++k) {
          const int h = warp * HPW + k;
          if (h < H && rg == 0) {
            const float inv = 1.f / ltot[k];
            T* o = out + ((size_t)b * H + h) * D + dl * DPV;
#pragma unroll
            for (int i = 0; i < DPV; ++i) o[i] = Elem<T>::from_f(acc[k][i] * inv);
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
              for (int i = 0; i < DPV; ++i) slot[dl * DPV + i] = acc[k][i];
            }
            if (lane == 0) {
              slot[D] = m[k];
              slot[D + 1] = ltot[k];
            }
          }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
          const int old = atomicAdd(&p.counters[b], 1);
          const int last = (old == nparts - 1);
          if (last) p.counters[b] = 0;  // every part has arrived; ready for the next call
          *flag = last;
        }
        __syncthreads();
        if (*flag) {
          __threadfence();
          for (int h = warp; h < H; h += nthreads / 32) {
            float M = -INFINITY;
            for (int cc = c_first; cc <= c_last; ++cc)
              M = fmaxf(M, __ldcg(p.partials + ((size_t)(b + cc) * H + h) * (D + 2) + D));
            float L = 0.f, o[DPV];
#pragma unroll
            for (int i = 0; i < DPV; ++i) o[i] = 0.f;
            for (int cc = c_first; cc <= c_last; ++cc) {
              const float* slot = p.partials + ((size_t)(b + cc) * H + h) * (D + 2);
              const float w = exp2f(__ldcg(slot + D) - M);
              L = fmaf(__ldcg(slot + D + 1), w, L);
#pragma unroll
              for (int i = 0; i < DPV; ++i) o[i] = fmaf(__ldcg(slot + dl * DPV + i), w, o[i]);
            }
            if (rg == 0) {
              const float inv = 1.f / L;
              T* op = out + ((size_t)b * H + h) * D + dl * DPV;
#pragma unroll
              for (int i = 0; i < DPV; ++i) op[i] = Elem<T>::from_f(o[i] * inv);
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

  if (abort_at >= 0 && tid == 0) {
    // A copy never completed: wait (bounded) for the copies still in flight, then leave.
    for (long long u = abort_at; u < issued; ++u) {
      (void)mbar_wait_bounded(&bars[(u - start) % S], (uint32_t)(((u - start) / S) & 1), nullptr);
    }
  }
}

// ------------------------------------------------------------------ host launcher
template <typename T, int D, int BS, int HPW>
static int launch_paged(const PagedParams& base, int device_sms, cudaStream_t stream) {
  PagedParams p = base;
  const int nw = (p.H + HPW - 1) / HPW;
  const int threads = nw * 32;
  const size_t stage_bytes = (size_t)2 * BS * p.H * D * sizeof(T);
  // Ring depth: enough stages for ~96 KB in flight, at least two when two fit.
  int S = (int)((96 * 1024) / stage_bytes);
  if (S < 2 && 2 * stage_bytes <= 200 * 1024) S = 2;
  S = S < 1 ? 1 : (S > 8 ? 8 : S);
  p.stages = S;
  const size_t smem = round_up((size_t)S * stage_bytes, 128) + 8 * (size_t)S + 4 * (2 * (size_t)p.B + 2);
  if (smem > 227 * 1024) return SPD_ERR_UNSUPPORTED;
  auto kfn = paged_decode_attn_kernel<T, D, BS, HPW>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return SPD_ERR_CUDA;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, threads, smem) != cudaSuccess || occ < 1)
    return SPD_ERR_CUDA;
  if (occ > kMaxCtasPerSm) occ = kMaxCtasPerSm;
  const int grid = device_sms * occ;
  kfn<<<grid, threads, smem, stream>>>(p);
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
