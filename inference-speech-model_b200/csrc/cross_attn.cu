// cross_attn.cu — op (2): single-query cross-attention over contiguous encoder K/V.
//
// Semantics follow speech_serving/models.py:167-203 (eager) and :468-479 (graph step):
//   out[b,h,:] = softmax_t( q[b,h,:]·K[b,h,t,:] * scale ) · V[b,h,t,:],  t < valid_b
// Positions at or beyond valid_b are excluded, which equals the reference's bool mask
// filled with finfo.min (models.py:196-197) and its additive -10000 fp16 mask
// (graph_decode_buffers.py:529): both drive exp() of those scores to exactly 0.
//
// B200 design (HBM-bound): a unit is a chunk of C consecutive positions of one
// (b, h) pair — C*D contiguous elements of K and of V — fetched with two 1-D bulk
// async copies (only valid rows).  Units of all pairs are laid end to end and each CTA
// of a persistent grid streams an equal share through an S-stage mbarrier ring.  Each
// warp keeps its own online-softmax state over the rows it reads; at the end of a pair
// the warps are merged in shared memory, and pairs split across CTAs are merged by the
// last CTA to arrive (arrival counter, no spinning).  The K/V stream is read under an L2
// evict-first policy and the split partials are stored evict-last, so the partials are
// still in L2 when the last CTA reads them back.
#include "spd_params.cuh"

namespace spd {

constexpr int kCrossComputeBarrier = 1;  // named barrier among compute warps

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

template <typename T, int D>
__global__ void __launch_bounds__(288) cross_attn_kernel(const CrossParams p) {
  using Gm = CrossGeom<T, D>;
  constexpr int NW = Gm::NW, LPR = Gm::LPR, RPP = Gm::RPP, DPL = Gm::DPL, CH = Gm::CH;
  constexpr int NCH = Gm::NCH, PASSES = Gm::PASSES, C = Gm::C;
  constexpr int PVL = Gm::PVL, PRG = Gm::PRG, DPV = Gm::DPV;
  constexpr int NCT = NW * 32;  // compute threads; warp NW is the producer

  extern __shared__ __align__(128) unsigned char smem[];
  const int H = p.H, B = p.B, S = p.stages;
  const size_t unit_elems = (size_t)C * D;
  const size_t stage_elems = 2 * unit_elems + D;  // K chunk, V chunk, q row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + round_up((size_t)S * stage_elems * sizeof(T), 128));
  uint64_t* empty = full + S;
  float* merge = reinterpret_cast<float*>(empty + S);          // [NW][D + 2]
  int* prefix = reinterpret_cast<int*>(merge + NW * (D + 2));  // [B + 1], units * H
  int* nch_s = prefix + B + 1;                                 // [B] chunks per pair
  int* val_s = nch_s + B;                                      // [B] clamped valid length
  int* flag = val_s + B;                                       // [0] last-arrival, [1] abort

  const T* __restrict__ kg = reinterpret_cast<const T*>(p.k);
  const T* __restrict__ vg = reinterpret_cast<const T*>(p.v);
  const T* __restrict__ qg = reinterpret_cast<const T*>(p.q);
  T* __restrict__ out = reinterpret_cast<T*>(p.out);

  // ---- 1. unit prefix: pair (b,h) has ceil(valid_b / C) units ----------------------
  for (int i = tid; i < B; i += blockDim.x) {
    int v = p.valid_lens[i];
    if (v > p.T_max) {
      set_error(p.err, SPD_DEVERR_LENGTH);
      v = p.T_max;
    }
    v = v > 0 ? v : 0;
    val_s[i] = v;
    nch_s[i] = (v + C - 1) / C;
    prefix[i + 1] = nch_s[i] * H;
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
  // Effective grid: never more CTAs than units (see paged_decode_attn.cu).
  const int c = blockIdx.x;
  const int G = (int)((long long)gridDim.x < W ? (long long)gridDim.x : W);
  for (int b = c; b < B; b += gridDim.x) {
    if (val_s[b] == 0) {
      for (int i = tid; i < H * D; i += blockDim.x) out[(size_t)b * H * D + i] = Elem<T>::from_f(0.f);
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
  __syncthreads();

  // ---- producer warp ---------------------------------------------------------------
  if (warp == NW) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
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
        const int off = (int)(u - prefix[pb]);
        const int h = off / nch_s[pb], j = off % nch_s[pb];
        const int nrows = min(C, val_s[pb] - j * C);
        const size_t src = (size_t)pb * p.kv_batch_stride + (size_t)h * p.kv_head_stride + (size_t)j * C * D;
        const uint32_t bytes = (uint32_t)(nrows * D * (int)sizeof(T));
        const bool seg_first = (u == start) || (j == 0);
        const uint32_t qbytes = seg_first ? (uint32_t)(D * sizeof(T)) : 0u;
        T* dst = ring + (size_t)s * stage_elems;
        mbar_arrive_expect_tx(&full[s], 2 * bytes + qbytes);
        bulk_copy_g2s_hint(dst, kg + src, bytes, &full[s], pol);
        bulk_copy_g2s_hint(dst + unit_elems, vg + src, bytes, &full[s], pol);
        if (seg_first) bulk_copy_g2s(dst + 2 * unit_elems, qg + ((size_t)pb * H + h) * D, qbytes, &full[s]);
        issued = u + 1;
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      const long long n = issued - start;
      for (int k = 0; k < S && k < n; ++k) {
        const long long u = issued - 1 - k;
        (void)mbar_wait_bounded(&full[(u - start) % S], (uint32_t)(((u - start) / S) & 1), nullptr);
      }
    }
    return;
  }

  // ---- compute warps -----------------------------------------------------------------
  const int r = lane / LPR, sub = lane % LPR, rot = r % NCH;
  const int dl = lane % PVL, rg = lane / PVL;
  float qr[DPL];
  float m = -INFINITY, l = 0.f, acc[DPV];

  int b = upper_index_i32(prefix, B, start);
  int h = (int)((start - prefix[b]) / nch_s[b]);
  bool need_q = true;
  int s = 0;
  uint32_t ph = 0;

  for (long long g = start; g < end; ++g) {
    const bool ok = !*((volatile int*)&flag[1]) && mbar_wait_bounded(&full[s], ph, p.err);
    if (!ok) flag[1] = 1;
    const int off = (int)(g - prefix[b]);
    const int j = off % nch_s[b];
    const int nrows = min(C, val_s[b] - j * C);
    const T* Ks = ring + (size_t)s * stage_elems;
    const T* Vs = Ks + unit_elems;
    if (need_q) {
      m = -INFINITY;
      l = 0.f;
#pragma unroll
      for (int i = 0; i < DPV; ++i) acc[i] = 0.f;
      const T* qrow = Vs + unit_elems + sub * DPL;  // q row arrived with this unit
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        const int ci = (cc + rot) % NCH;
#pragma unroll
        for (int e = 0; e < CH; ++e) qr[cc * CH + e] = ok ? Elem<T>::to_f(qrow[ci * CH + e]) * p.scale_log2 : 0.f;
      }
      need_q = false;
    }
    if (ok) {
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
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }

    const bool seg_end = (j == nch_s[b] - 1);
    if (seg_end || g + 1 == end) {
      // merge the compute warps' states for pair (b, h)
      float lw = warp_sum(l);
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
      const long long pair = (long long)b * H + h;
      const long long u0 = prefix[b] + (long long)h * nch_s[b];
      const long long u1 = u0 + nch_s[b];
      const bool whole = (start <= u0) && (end >= u1);
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
      if (whole) {
        if (warp == 0 && rg == 0) {
          const float inv = 1.f / L;
          T* op = out + (size_t)pair * D + dl * DPV;
#pragma unroll
          for (int i = 0; i < DPV; ++i) op[i] = Elem<T>::from_f(o[i] * inv);
        }
      } else {
        const int c_first = cta_of_unit(u0, G, W);
        const int c_last = cta_of_unit(u1 - 1, G, W);
        const int nparts = c_last - c_first + 1;
        float* slot = p.partials + (size_t)(pair + c) * (D + 2);
        if (warp == 0) {
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
        named_sync(kCrossComputeBarrier, NCT);
        if (tid == 0) {
          __threadfence();
          const int old = atomicAdd(&p.counters[pair], 1);
          const int last = (old == nparts - 1);
          if (last) {
            p.counters[pair] = 0;
            __threadfence();
          }
          flag[0] = last;
        }
        named_sync(kCrossComputeBarrier, NCT);
        if (flag[0] && warp == 0) {
          float M2 = -INFINITY;
          for (int cc = c_first; cc <= c_last; ++cc)
            M2 = fmaxf(M2, __ldcg(p.partials + (size_t)(pair + cc) * (D + 2) + D));
          float L2 = 0.f, o2[DPV];
#pragma unroll
          for (int i = 0; i < DPV; ++i) o2[i] = 0.f;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const float* sl = p.partials + (size_t)(pair + cc) * (D + 2);
            const float wt = exp2f(__ldcg(sl + D) - M2);
            L2 = fmaf(__ldcg(sl + D + 1), wt, L2);
#pragma unroll
            for (int i = 0; i < DPV; ++i) o2[i] = fmaf(__ldcg(sl + dl * DPV + i), wt, o2[i]);
          }
          if (rg == 0) {
            const float inv = 1.f / L2;
            T* op = out + (size_t)pair * D + dl * DPV;
#pragma unroll
            for (int i = 0; i < DPV; ++i) op[i] = Elem<T>::from_f(o2[i] * inv);
          }
        }
      }
      named_sync(kCrossComputeBarrier, NCT);  // merge buffer is reused by the next pair
      if (seg_end) {
        ++h;
        if (h == H) {
          h = 0;
          ++b;
          while (b < B && nch_s[b] == 0) ++b;
        }
        need_q = true;
      }
    }
  }
}

template <typename T, int D>
static int launch_cross(const CrossParams& base, int sms, cudaStream_t stream) {
  using Gm = CrossGeom<T, D>;
  CrossParams p = base;
  const size_t stage_bytes = ((size_t)2 * Gm::C + 1) * D * sizeof(T);
  // ~96 KB of stages per CTA: two CTAs per SM, each with a producer warp streaming.
  int S = (int)((96 * 1024) / stage_bytes);
  S = S < 2 ? 2 : (S > 8 ? 8 : S);
  p.stages = S;
  const size_t smem = round_up((size_t)S * stage_bytes, 128) + 16 * (size_t)S +
                      4 * (size_t)Gm::NW * (D + 2) + 4 * (3 * (size_t)p.B + 3);
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
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
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
