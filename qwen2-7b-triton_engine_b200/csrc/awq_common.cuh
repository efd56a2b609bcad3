// awq_common.cuh -- shared device helpers for the sm_100a AWQ W4A16 kernels.
//
// Packed layout (songqiuyu/Qwen2-7B-Triton_Engine, model/qwen2.py:34-36 and
// kernels/awq_gemm.py:36-38):
//   qweight int32 [K, N/8]   element n of row k is nibble order[n % 8] of word
//                            qweight[k, n / 8], order = [0,4,1,5,2,6,3,7];
//                            equivalently nibble slot j holds element
//                            [0,2,4,6,1,3,5,7][j]
//   qzeros  int32 [K/gs, N/8] same packing, one row per group of gs rows
//   scales  fp16  [K/gs, N]
//   W[k, n] = (fp16(w) - fp16(z)) * scale, rounded once to fp16 (awq_gemm.py:59)
//
// Unpack used by every kernel here.  Because slot j holds element 2j for j < 4
// and element 2j-7 for j >= 4, the two nibbles of a 16-bit half of a word at
// bit offsets (4i, 16 + 4i) are the element pair (2i, 2i+1).  OR-ing the masked
// word into 0x6400 (fp16 1024.0, whose ulp is 1) turns nibble v at bits 0..3 into
// the fp16 value 1024 + v and nibble v at bits 4..7 into 1024 + 16 v, both
// exact.  One subtraction (bits 0..3) or one fma with 1/16 (bits 4..7) then
// yields the exact small integer w - z, and a single fp16 multiply by the scale
// rounds exactly like the reference's fp16 (w - z) * scale.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace awq {

// Error flag bits written by kernels into the library's device status word.
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrBarrierTimeout = 1,   // an mbarrier wait gave up (bounded spin)
  kDevErrShape = 2,            // a kernel saw parameters it cannot handle
  kDevErrPeerTimeout = 4,      // a wait for other ranks' all-reduce contributions gave up
};

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (a & mask) | orv  -- lut: (0xF0 & 0xCC) | 0xAA = 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}
// Same with compile-time mask and OR value (immediate operands, no register needed).
template <uint32_t MASK, uint32_t ORV>
__device__ __forceinline__ uint32_t lop3_and_or_imm(uint32_t a) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "n"(MASK), "n"(ORV));
  return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

constexpr uint32_t kMagic = 0x64006400u;       // half2(1024, 1024)
constexpr uint32_t kLoMask = 0x000F000Fu;
constexpr uint32_t kHiMask = 0x00F000F0u;
constexpr uint32_t kInv16 = 0x2C002C00u;       // half2(1/16, 1/16)
constexpr uint32_t kNegInv16 = 0xAC00AC00u;    // half2(-1/16, -1/16)

// Per-group zero constants for one packed zero word:
//   zc[0] = (1024 + z0, 1024 + z1)   subtracted from the bits 0..3 path
//   zc[1] = (-(64 + z2), -(64 + z3)) added by the fma of the bits 4..7 path
//   zc[2] = (1024 + z4, 1024 + z5)
//   zc[3] = (-(64 + z6), -(64 + z7))
__device__ __forceinline__ void zero_consts(uint32_t zw, uint32_t zc[4]) {
  uint32_t z8 = zw >> 8;
  zc[0] = lop3_and_or(zw, kLoMask, kMagic);
  zc[1] = hmul2_u32(lop3_and_or(zw, kHiMask, kMagic), kNegInv16);   // exact: power of two
  zc[2] = lop3_and_or(z8, kLoMask, kMagic);
  zc[3] = hmul2_u32(lop3_and_or(z8, kHiMask, kMagic), kNegInv16);
}

// Exact (w - z) for the 8 elements of one packed word, as 4 half2 pairs
// (e0,e1), (e2,e3), (e4,e5), (e6,e7).
__device__ __forceinline__ void unpack_minus_zero(uint32_t w, const uint32_t zc[4], uint32_t d[4]) {
  uint32_t w8 = w >> 8;
  d[0] = hsub2_u32(lop3_and_or(w, kLoMask, kMagic), zc[0]);
  d[1] = hfma2_u32(lop3_and_or(w, kHiMask, kMagic), kInv16, zc[1]);
  d[2] = hsub2_u32(lop3_and_or(w8, kLoMask, kMagic), zc[2]);
  d[3] = hfma2_u32(lop3_and_or(w8, kHiMask, kMagic), kInv16, zc[3]);
}

// Bit-exact dequant of one packed word: W = fp16((w - z) * s) for 8 elements.
// s[j] holds the scales of elements (2j, 2j+1).
__device__ __forceinline__ void dequant_word(uint32_t w, const uint32_t zc[4], const uint32_t s[4],
                                             uint32_t d[4]) {
  unpack_minus_zero(w, zc, d);
#pragma unroll
  for (int j = 0; j < 4; ++j) d[j] = hmul2_u32(d[j], s[j]);
}

// ---------------------------------------------------------------------------------
// Global memory helpers
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

}  // namespace awq
