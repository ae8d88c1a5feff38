// decoder_layer_ops.cu — the residual add fused with the LayerNorm that follows it, for
// the decoder layers' glue between the decode-path kernels.
//
// A Whisper decoder layer ends each sub-block with `x = x + sublayer(...)` and starts
// the next with `LayerNorm(x)` (speech_serving/models.py:163-207; transformers
// WhisperDecoderLayer).  In a batch-64 decode step these are ~100 tiny launches; here
// one warp per row does both:
//   x_out[r] = round_T(x[r] + delta[r])                 (delta may be null)
//   y[r]     = round_T((x_out[r] - mean) * rstd * gamma + beta),  rstd = (var + eps)^-1/2
// The statistics are taken from the rounded x_out, as when the add and the LayerNorm
// run one after the other in the model dtype, and accumulate in fp32 (two passes over
// the row held in registers).  x_out may alias x.
//
// Both kernels here are launched with programmatic dependent launch: they signal
// launch_dependents on entry, so a PDL-launched kernel behind them (the small-batch GEMM
// that consumes the LayerNorm output) gets resident and prefetches its weights while
// they run.  Every input, parameters included, is read after griddepcontrol.wait, so
// results never depend on what the kernel before them writes.
#include "spd_params.cuh"

namespace spd {

// Launches kfn(args) on `st` with programmatic stream serialization allowed.
template <typename K, typename... Args>
static int launch_pdl(K kfn, dim3 grid, dim3 block, cudaStream_t st, const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kfn, args...) == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
}

// VPL: 16-byte vectors per lane (a row of up to 32 * VPL vectors).
template <typename T, int VPL>
__global__ void __launch_bounds__(128) add_layernorm_kernel(const AddLnParams p) {
  constexpr int E = 16 / sizeof(T);  // elements per vector
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= p.rows) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  const int nvec = p.cols / E;
  const T* x = reinterpret_cast<const T*>(p.x) + row * p.cols;
  const T* dl = p.delta ? reinterpret_cast<const T*>(p.delta) + row * p.cols : nullptr;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x, delta, gamma, beta: written before this kernel
  // gamma and beta do not depend on the row: with few vectors per lane they are loaded up
  // front, so their latency overlaps the row's loads and reductions instead of following them
  constexpr bool kPrefetch = VPL <= 4;
  uint4 gpre[kPrefetch ? VPL : 1], bpre[kPrefetch ? VPL : 1];
  if constexpr (kPrefetch) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        gpre[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.gamma) + vi * E);
        bpre[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.beta) + vi * E);
      }
    }
  }
  float v[VPL][E];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      const uint4 a = *reinterpret_cast<const uint4*>(x + vi * E);
      const T* ae = reinterpret_cast<const T*>(&a);
      if (dl) {
        const uint4 d = *reinterpret_cast<const uint4*>(dl + vi * E);
        const T* de = reinterpret_cast<const T*>(&d);
#pragma unroll
        for (int k = 0; k < E; ++k) v[i][k] = Elem<T>::to_f(Elem<T>::from_f(Elem<T>::to_f(ae[k]) + Elem<T>::to_f(de[k])));
      } else {
#pragma unroll
        for (int k = 0; k < E; ++k) v[i][k] = Elem<T>::to_f(ae[k]);
      }
#pragma unroll
      for (int k = 0; k < E; ++k) sum += v[i][k];
    }
  }
  const float mean = warp_sum(sum) / (float)p.cols;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (lane + 32 * i < nvec)
#pragma unroll
      for (int k = 0; k < E; ++k) {
        const float c = v[i][k] - mean;
        sq += c * c;
      }
  const float rstd = rsqrtf(warp_sum(sq) / (float)p.cols + p.eps);
  const T* g = reinterpret_cast<const T*>(p.gamma);
  const T* bt = reinterpret_cast<const T*>(p.beta);
  T* xo = reinterpret_cast<T*>(p.x_out) + row * p.cols;
  T* y = reinterpret_cast<T*>(p.y) + row * p.y_ld;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi >= nvec) continue;
    uint4 gv, bv;
    if constexpr (kPrefetch) {
      gv = gpre[i];
      bv = bpre[i];
    } else {
      gv = *reinterpret_cast<const uint4*>(g + vi * E);
      bv = *reinterpret_cast<const uint4*>(bt + vi * E);
    }
    const T* ge = reinterpret_cast<const T*>(&gv);
    const T* be = reinterpret_cast<const T*>(&bv);
    alignas(16) T o[E];
    alignas(16) T s[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
      o[k] = Elem<T>::from_f((v[i][k] - mean) * rstd * Elem<T>::to_f(ge[k]) + Elem<T>::to_f(be[k]));
      s[k] = Elem<T>::from_f(v[i][k]);
    }
    if (dl) *reinterpret_cast<uint4*>(xo + vi * E) = *reinterpret_cast<const uint4*>(s);
    *reinterpret_cast<uint4*>(y + vi * E) = *reinterpret_cast<const uint4*>(o);
  }
}

template <typename T>
static int add_ln_dispatch(const AddLnParams& p, cudaStream_t st) {
  constexpr int E = 16 / sizeof(T);
  const int nvec = p.cols / E;
  const int vpl = (nvec + 31) / 32;
  // four rows per CTA: a decode step's few rows spread over more SMs
  const unsigned grid = (unsigned)((p.rows + 3) / 4);
  auto run = [&](auto kfn) { return launch_pdl(kfn, dim3(grid), dim3(128), st, p); };
  switch (vpl) {
    case 1: return run(add_layernorm_kernel<T, 1>);
    case 2: return run(add_layernorm_kernel<T, 2>);
    case 3: return run(add_layernorm_kernel<T, 3>);
    case 4: return run(add_layernorm_kernel<T, 4>);
    case 5: case 6: return run(add_layernorm_kernel<T, 6>);
    case 7: case 8: return run(add_layernorm_kernel<T, 8>);
    default:
      if constexpr (sizeof(T) == 4) {  // fp32 rows of up to 2048 elements
        if (vpl <= 12) return run(add_layernorm_kernel<T, 12>);
        if (vpl <= 16) return run(add_layernorm_kernel<T, 16>);
      }
      return SPD_ERR_UNSUPPORTED;
  }
}

// ------------------------------------------------------------------ greedy token pick
// out[r] = argmax_c x[r][c] over c < cols, a column with skip[c] != 0 counting as -inf:
// the same index as torch.argmax(x.masked_fill(skip, -inf), dim=-1), i.e. the first
// maximal column, and the first NaN when a row holds one (the reference's greedy step,
// speech_serving/models.py:598-610: suppress mask, then argmax over the vocabulary).
// One CTA per row; each thread scans 16-byte vectors, then the CTA reduces (value, index).
struct ArgBest {
  float v;
  int i;
};

// a beats b: NaN over numbers, larger value, then the lower index
__device__ __forceinline__ bool arg_better(float av, int ai, float bv, int bi) {
  const bool an = av != av, bn = bv != bv;
  if (an || bn) return an && (!bn || ai < bi);
  return av > bv || (av == bv && ai < bi);
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const ArgmaxParams p) {
  constexpr int E = 16 / sizeof(T);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the logits come from the previous kernel
  const T* x = reinterpret_cast<const T*>(p.x) + (long long)blockIdx.x * p.ld;
  const unsigned char* skip = reinterpret_cast<const unsigned char*>(p.skip);
  ArgBest best{-INFINITY, 0x7fffffff};
  auto consider = [&](float v, int c) {
    if (skip && skip[c]) v = -INFINITY;
    if (arg_better(v, c, best.v, best.i)) best = ArgBest{v, c};
  };
  if (p.vec) {
    // four vectors per thread in flight per round (a row is read once, from L2 or DRAM)
    constexpr int U = 4;
    const int step = (int)blockDim.x * E;
    for (int c0 = threadIdx.x * E; c0 < p.cols; c0 += U * step) {
      uint4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * step;
        if (c + E <= p.cols) w[u] = *reinterpret_cast<const uint4*>(x + c);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * step;
        if (c + E <= p.cols) {
          const T* e = reinterpret_cast<const T*>(&w[u]);
#pragma unroll
          for (int k = 0; k < E; ++k) consider(Elem<T>::to_f(e[k]), c + k);
        } else {
          for (int cc = c; cc < p.cols; ++cc) consider(Elem<T>::to_f(x[cc]), cc);
        }
      }
    }
  } else {
    for (int c = threadIdx.x; c < p.cols; c += blockDim.x) consider(Elem<T>::to_f(x[c]), c);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
    if (arg_better(ov, oi, best.v, best.i)) best = ArgBest{ov, oi};
  }
  __shared__ ArgBest warp_best[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_best[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (int)(blockDim.x >> 5) ? warp_best[lane] : ArgBest{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
      if (arg_better(ov, oi, best.v, best.i)) best = ArgBest{ov, oi};
    }
    if (lane == 0) p.out[blockIdx.x] = best.i;
  }
}

int argmax_rows_launch(const ArgmaxParams& p, int dtype, cudaStream_t st) {
  const unsigned threads = p.cols >= 8192 ? 1024u : 256u;
  switch (dtype) {
    case SPD_F32: return launch_pdl(argmax_rows_kernel<float>, dim3(p.rows), dim3(threads), st, p);
    case SPD_F16: return launch_pdl(argmax_rows_kernel<__half>, dim3(p.rows), dim3(threads), st, p);
    case SPD_BF16: return launch_pdl(argmax_rows_kernel<__nv_bfloat16>, dim3(p.rows), dim3(threads), st, p);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

int add_layernorm_launch(const AddLnParams& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case SPD_F32: return add_ln_dispatch<float>(p, st);
    case SPD_F16: return add_ln_dispatch<__half>(p, st);
    case SPD_BF16: return add_ln_dispatch<__nv_bfloat16>(p, st);
    default: return SPD_ERR_UNSUPPORTED;
  }
}

}  // namespace spd
