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
#include "spd_params.cuh"

namespace spd {

// VPL: 16-byte vectors per lane (a row of up to 32 * VPL vectors).
template <typename T, int VPL>
__global__ void __launch_bounds__(256) add_layernorm_kernel(const AddLnParams p) {
  constexpr int E = 16 / sizeof(T);  // elements per vector
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nvec = p.cols / E;
  const T* x = reinterpret_cast<const T*>(p.x) + row * p.cols;
  const T* dl = p.delta ? reinterpret_cast<const T*>(p.delta) + row * p.cols : nullptr;
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
  T* y = reinterpret_cast<T*>(p.y) + row * p.cols;
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
  const unsigned grid = (unsigned)((p.rows + 7) / 8);
  switch (vpl) {
    case 1: add_layernorm_kernel<T, 1><<<grid, 256, 0, st>>>(p); break;
    case 2: add_layernorm_kernel<T, 2><<<grid, 256, 0, st>>>(p); break;
    case 3: add_layernorm_kernel<T, 3><<<grid, 256, 0, st>>>(p); break;
    case 4: add_layernorm_kernel<T, 4><<<grid, 256, 0, st>>>(p); break;
    case 5: case 6: add_layernorm_kernel<T, 6><<<grid, 256, 0, st>>>(p); break;
    case 7: case 8: add_layernorm_kernel<T, 8><<<grid, 256, 0, st>>>(p); break;
    default:
      if constexpr (sizeof(T) == 4) {  // fp32 rows of up to 2048 elements
        if (vpl <= 12) {
          add_layernorm_kernel<T, 12><<<grid, 256, 0, st>>>(p);
          break;
        }
        if (vpl <= 16) {
          add_layernorm_kernel<T, 16><<<grid, 256, 0, st>>>(p);
          break;
        }
      }
      return SPD_ERR_UNSUPPORTED;
  }
  return cudaPeekAtLastError() == cudaSuccess ? SPD_OK : SPD_ERR_CUDA;
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
