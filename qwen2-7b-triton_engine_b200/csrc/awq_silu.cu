// awq_silu.cu -- SiLU-mul of the fused gate+up product, for the calls whose product kernel
// cannot fuse it into its epilogue (awq_gemm_f16_silu_mul above 8 tokens, or gate / up
// halves that do not split at a 256-column strip).
//
// Same arithmetic as the reference's _silu_mul_kernel (songqiuyu/Qwen2-7B-Triton_Engine
// kernels/silu_mul.py:41-64) on the two halves that model/qwen2.py:183-188 slices out of
// the gate+up product: fp16 inputs widened to fp32, x * sigmoid(x) * y, rounded once to
// fp16.  Here the halves are read in place (no .contiguous() copies).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "awq_common.cuh"
#include "awq_internal.h"

namespace awq {

namespace {

__device__ __forceinline__ float silu_mul1(__half g, __half u) {
  const float x = __half2float(g), y = __half2float(u);
  return x * (1.0f / (1.0f + expf(-x))) * y;
}

// 8 columns per thread with 16-byte loads and stores (I, ldg, ldo multiples of 8 and
// 16-byte aligned rows), grid-stride.
__global__ void __launch_bounds__(256)
silu_mul_vec8(const __half* __restrict__ gu, int64_t ldg, int M, int I, __half* __restrict__ out,
              int64_t ldo) {
  const int per_row = I / 8;
  const int64_t total = (int64_t)M * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / per_row;
    const int c = (int)(i - m * per_row) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + m * ldg + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + m * ldg + I + c);
    const __half* g = reinterpret_cast<const __half*>(&gv);
    const __half* u = reinterpret_cast<const __half*>(&uv);
    uint4 ov;
    __half* o = reinterpret_cast<__half*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(silu_mul1(g[j], u[j]));
    *reinterpret_cast<uint4*>(out + m * ldo + c) = ov;
  }
}

__global__ void __launch_bounds__(256)
silu_mul_scalar(const __half* __restrict__ gu, int64_t ldg, int M, int I,
                __half* __restrict__ out, int64_t ldo) {
  const int64_t total = (int64_t)M * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / I;
    const int n = (int)(i - m * I);
    out[m * ldo + n] = __float2half_rn(silu_mul1(gu[m * ldg + n], gu[m * ldg + I + n]));
  }
}

}  // namespace

cudaError_t launch_silu_mul(const void* gu, int64_t ldg, int M, int I, void* out, int64_t ldo,
                            int num_sms, cudaStream_t stream) {
  if (M <= 0 || I <= 0) return cudaSuccess;
  const bool vec = I % 8 == 0 && ldg % 8 == 0 && ldo % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(gu) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const int64_t work = vec ? (int64_t)M * (I / 8) : (int64_t)M * I;
  int64_t blocks = (work + 255) / 256;
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (vec)
    silu_mul_vec8<<<(int)blocks, 256, 0, stream>>>(static_cast<const __half*>(gu), ldg, M, I,
                                                   static_cast<__half*>(out), ldo);
  else
    silu_mul_scalar<<<(int)blocks, 256, 0, stream>>>(static_cast<const __half*>(gu), ldg, M, I,
                                                     static_cast<__half*>(out), ldo);
  return cudaGetLastError();
}

}  // namespace awq
