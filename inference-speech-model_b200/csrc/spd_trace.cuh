// spd_trace.cuh — optional %globaltimer timeline of one launch, for trace builds only.
//
// A trace build (csrc/build.py --trace, library lib/libspd_b200_trace.so) compiles the
// kernels with SPD_TRACE_BUILD defined: each marked point of each CTA stores the
// %globaltimer value into a file-scope device array, [kernel][CTA][point]; every launch
// overwrites the previous one's values, so the array holds the last launch.  The normal
// build compiles every mark to nothing.  The arrays are per translation unit: the file
// that marks points also exports the function that copies them out.
#pragma once

#include "spd_common.cuh"

namespace spd {
constexpr int kTraceCtas = 1024;  // CTAs recorded per kernel (blockIdx.x modulo this)
constexpr int kTracePoints = 12;  // marks per CTA
constexpr int kTraceKernels = 2;  // streaming kernel, merge kernel
}  // namespace spd

#ifdef SPD_TRACE_BUILD
#define SPD_TRACE_ARRAY                                                                          \
  namespace spd {                                                                                \
  static __device__ unsigned long long g_trace[kTraceKernels * kTraceCtas * kTracePoints];       \
  }
#define SPD_TRACE_AT(kernel, point) SPD_TRACE_VALUE(kernel, point, spd::global_ns())
#define SPD_TRACE_VALUE(kernel, point, value)                                                    \
  (spd::g_trace[((kernel) * spd::kTraceCtas + (blockIdx.x % spd::kTraceCtas)) * spd::kTracePoints + \
                (point)] = (unsigned long long)(value))
#else
#define SPD_TRACE_ARRAY
#define SPD_TRACE_AT(kernel, point) ((void)0)
#define SPD_TRACE_VALUE(kernel, point, value) ((void)0)
#endif
