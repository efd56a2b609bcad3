// awq_gemm_tc.cu -- placeholder until the tcgen05 prefill kernel lands.
#include "awq_internal.h"

namespace awq {

bool tc_supported(const void*, int64_t, const int32_t*, const int32_t*, const void*, int64_t,
                  int64_t, int64_t, int64_t) {
  return false;
}

cudaError_t launch_gemm_tc(const void*, int64_t, const int32_t*, const int32_t*, const void*,
                           void*, int64_t, int, int, int, int, int, int*, cudaStream_t,
                           const char** why) {
  *why = "not built";
  return cudaSuccess;
}

}  // namespace awq
