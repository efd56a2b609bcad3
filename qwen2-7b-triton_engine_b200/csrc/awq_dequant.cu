// awq_dequant.cu -- bit-exact AWQ int4 -> fp16 dequantization on sm_100a.
//
// Replaces _dequant_awq_kernel / _dequant_to_fp16
// (songqiuyu/Qwen2-7B-Triton_Engine, kernels/awq_gemm.py:14-87).  Output W[k, n]
// equals the reference's fp16 (w - z) * scale bit for bit (see awq_common.cuh for
// the unpack and the rounding argument).
//
// Pure streaming transform: 0.5 B (qweight) + 2 B (W) per element, plus the
// per-group zeros/scales that stay in L2.  Each thread handles one packed word
// (8 outputs, one 16-byte store) or, when rows are 16-byte aligned, four
// consecutive words (one 16-byte load, four 16-byte stores).  The grid is a
// grid-stride loop sized to a whole number of waves over the SMs.
#include "awq_common.cuh"
#include "awq_internal.h"

namespace awq {

template <bool VEC4>
__global__ void __launch_bounds__(256) dequant_kernel(const int32_t* __restrict__ qweight,
                                                      const int32_t* __restrict__ qzeros,
                                                      const __half* __restrict__ scales,
                                                      __half* __restrict__ out, int64_t K,
                                                      int64_t PN, int group_size) {
  constexpr int WPT = VEC4 ? 4 : 1;                 // packed words per thread
  const int64_t PNv = PN / WPT;
  const int64_t total = K * PNv;
  const int64_t N = PN * 8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = idx / PNv;
    const int64_t wv = idx - k * PNv;
    const int64_t grp = k / group_size;
    uint32_t w[WPT], z[WPT];
    if constexpr (VEC4) {
      uint4 q = ldg_stream_v4(qweight + k * PN + wv * 4);
      uint4 qz = *reinterpret_cast<const uint4*>(qzeros + grp * PN + wv * 4);
      w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
      z[0] = qz.x; z[1] = qz.y; z[2] = qz.z; z[3] = qz.w;
    } else {
      w[0] = ldg_stream_u32(qweight + k * PN + wv);
      z[0] = static_cast<uint32_t>(qzeros[grp * PN + wv]);
    }
#pragma unroll
    for (int c = 0; c < WPT; ++c) {
      const int64_t n0 = (wv * WPT + c) * 8;
      uint4 s4 = *reinterpret_cast<const uint4*>(scales + grp * N + n0);
      uint32_t s[4] = {s4.x, s4.y, s4.z, s4.w};
      uint32_t zc[4], d[4];
      zero_consts(z[c], zc);
      dequant_word(w[c], zc, s, d);
      *reinterpret_cast<uint4*>(out + k * N + n0) = make_uint4(d[0], d[1], d[2], d[3]);
    }
  }
}

cudaError_t launch_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales,
                           void* out, int64_t K, int64_t N, int64_t group_size, int num_sms,
                           cudaStream_t stream) {
  const int64_t PN = N / 8;
  const bool vec4 = (PN % 4 == 0) && ((reinterpret_cast<uintptr_t>(qweight) & 15) == 0) &&
                    ((reinterpret_cast<uintptr_t>(qzeros) & 15) == 0);
  const int64_t items = vec4 ? K * (PN / 4) : K * PN;
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms * 8;            // 8 CTAs of 256 threads per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const __half* s = static_cast<const __half*>(scales);
  __half* o = static_cast<__half*>(out);
  if (vec4)
    dequant_kernel<true><<<(unsigned)blocks, threads, 0, stream>>>(qweight, qzeros, s, o, K, PN,
                                                                 (int)group_size);
  else
    dequant_kernel<false><<<(unsigned)blocks, threads, 0, stream>>>(qweight, qzeros, s, o, K, PN,
                                                                  (int)group_size);
  return cudaGetLastError();
}

}  // namespace awq
