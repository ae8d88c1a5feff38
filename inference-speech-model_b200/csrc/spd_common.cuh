// spd_common.cuh — device helpers shared by the decode-path kernels (sm_100a).
//
// - element conversion for fp32 / fp16 / bf16 storage with fp32 arithmetic;
// - 1-D bulk async copies (cp.async.bulk, no multicast) completing on an mbarrier;
// - bounded mbarrier waits: every wait gives up after SPD_WAIT_NS of wall time, records
//   SPD_DEVERR_TIMEOUT in the launch's error word and lets the kernel return;
// - the error word helpers and the workspace header layout.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/spd_b200.h"

namespace spd {

// Workspace layout (bytes): [0,256) header (int32 error word at 0, work-queue counters at
// 128), then a [B*H] int region, then fp32 partial slots.  Sizes are rounded to 256 bytes.
constexpr size_t kWsHeaderBytes = 256;
// Upper bound on resident CTAs per SM that any attention launch uses.
constexpr int kMaxCtasPerSm = 4;
// Paged attention work item: up to this many consecutive pool blocks of one sequence.
constexpr int kItemUnits = 2;
// Cross-attention work items per (b, h) pair at most (sizes its partial slots).
constexpr int kCrossMaxItems = 6;
// Block tables up to this size are bulk-copied into each CTA's shared memory.
constexpr size_t kTableSmemMax = 16384;
// Workspace header: error word at byte 0, the attention kernels' work-queue counters at
// byte 128.
constexpr size_t kWsWorkOffset = 128;
// Bounded wait: 2 s of %globaltimer.
constexpr unsigned long long SPD_WAIT_NS = 2000000000ull;

__host__ __device__ inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------- element conversion
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Converts `n` consecutive elements at p (in shared or global memory, 4-byte aligned
// for 16-bit types) to fp32.  n is a compile-time constant so the loop unrolls.
template <typename T, int N>
__device__ __forceinline__ void load_to_float(const T* p, float* out) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        float4 v = *reinterpret_cast<const float4*>(p + i);
        out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
      }
    } else if constexpr (N % 2 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        float2 v = *reinterpret_cast<const float2*>(p + i);
        out[i] = v.x; out[i + 1] = v.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = p[i];
    }
  } else {
    // 16-bit: move 16/8/4 bytes at a time, then unpack pairs.
    if constexpr (N % 8 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 8) {
        uint4 v = *reinterpret_cast<const uint4*>(p + i);
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) out[i + k] = Elem<T>::to_f(e[k]);
      }
    } else if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        uint2 v = *reinterpret_cast<const uint2*>(p + i);
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) out[i + k] = Elem<T>::to_f(e[k]);
      }
    } else if constexpr (N % 2 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        uint32_t v = *reinterpret_cast<const uint32_t*>(p + i);
        const T* e = reinterpret_cast<const T*>(&v);
        out[i] = Elem<T>::to_f(e[0]);
        out[i + 1] = Elem<T>::to_f(e[1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = Elem<T>::to_f(p[i]);
    }
  }
}

// ---------------------------------------------------------------- error word
__device__ __forceinline__ void set_error(int* word, int flag) {
  if (word) atomicOr(word, flag);
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's prior generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// L2 policy for data read once per launch (the K/V stream): its lines are the first to
// be evicted, so the small inputs, partials and code that the next launch reads again
// stay resident in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 policy for data the next kernel reads back (split partials): kept over the stream.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 8- and 16-byte global stores with an L2 cache policy.
__device__ __forceinline__ void st_global_hint(float* p, float2 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(v.x), "f"(v.y), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void st_global_hint(float* p, float4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w), "l"(policy)
               : "memory");
}

// As bulk_copy_g2s, with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_copy_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 1-D bulk async copy global -> shared (no multicast).  dst, src 16-byte aligned,
// bytes a multiple of 16.  Completion is signalled as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of `bar` to complete.  Returns false (and sets the
// timeout flag) if it did not complete within `limit_ns` (SPD_WAIT_NS by default).  The
// attention kernels pass the launch's limit (spd_set_wait_timeout_ns) to the waits that
// make progress; the waits that drain copies still in flight before a CTA exits keep the
// default, so that shared memory is never released under a copy.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  unsigned long long limit_ns = SPD_WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  // the clock is read every 64 tries: a read per try slows spinning warps enough to be
  // measurable in the serving loop (kernels spinning beside others on the same SMs)
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && global_ns() - t0 > limit_ns) {
      set_error(err, SPD_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// 2^x by the hardware approximation (ex2.approx.ftz: results below 2^-126 are 0, which for
// softmax weights relative to the running maximum is exact enough); 2^-inf = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Hint: bring [src, src + bytes) of global memory into L2 (no completion, no data
// returned; src 16-byte aligned, bytes a multiple of 16).  Because it only warms L2, which
// is coherent for the whole device, it is safe on addresses whose contents another kernel
// may still be writing.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 32-bit shared-memory load (a pair of 16-bit elements), for tensor-core fragments.
__device__ __forceinline__ uint32_t lds_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// D += A·B on the tensor cores, m16n8k16, 16-bit inputs (T = __half or __nv_bfloat16),
// fp32 accumulation; fragments in the PTX ISA's register layout for mma.m16n8k16.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// ---------------------------------------------------------------- warp reductions
// Maximum over the warp in one instruction (sm_100a redux.sync on fp32).
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- stream partition
// Units (pool blocks or K/V chunks) of all segments are laid end to end; CTA c of G
// streams units [c*W/G, (c+1)*W/G).  Unit p belongs to CTA ceil((p+1)*G/W) - 1.
__device__ __forceinline__ long long range_start(int c, int G, long long W) {
  return (long long)c * W / G;
}
__device__ __forceinline__ int cta_of_unit(long long p, int G, long long W) {
  return (int)(((p + 1) * (long long)G + W - 1) / W) - 1;
}

// Largest index i in [0, n] with prefix[i] <= x (prefix non-decreasing, prefix[0] = 0).
// With x < prefix[n] the result is the non-empty segment that contains unit x.
__device__ __forceinline__ int upper_index_i32(const int* prefix, int n, long long x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

}  // namespace spd
