// cross_kv_project.cu — op (4): cross-KV projection GEMM at encoder handoff
// (speech_serving/models.py:554-561).  The tcgen05 implementation is added in this
// file; until it is present the entry point reports SPD_ERR_UNSUPPORTED.
#include "spd_params.cuh"

namespace spd {

int cross_kv_project_launch(const void*, const void*, const void*, void*, const int32_t*, int, int, int, int,
                            int, int, int, int64_t, int, int*, int, cudaStream_t) {
  return SPD_ERR_UNSUPPORTED;
}

}  // namespace spd
