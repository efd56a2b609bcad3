/*
 * awq_oracle.c -- CPU restatement of the reference's AWQ W4A16 path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it.  The product path never calls it.
 *
 * What it restates (file:line are paths inside songqiuyu/Qwen2-7B-Triton_Engine):
 *   - kernels/awq_gemm.py:36-38   nibble position of element e = n % 8 inside a
 *                                 packed int32: shift = 4 * order[e],
 *                                 order = [0,4,1,5,2,6,3,7]
 *   - kernels/awq_gemm.py:46,52   w = (qweight >> shift) & 0xF,
 *                                 z = (qzeros  >> shift) & 0xF
 *   - kernels/awq_gemm.py:49,55   scale row = k / group_size
 *   - kernels/awq_gemm.py:59      W = (fp16(w) - fp16(z)) * scale, in fp16
 *   - kernels/awq_gemm.py:266     out = x @ W (the M<=4 branch; the oracle
 *                                 accumulates in fp32 like x.float() @ W.float())
 *
 * Bit-exactness argument: fp16(w) - fp16(z) is an exact integer in [-15, 15];
 * its product with an fp16 scale needs at most 4 + 11 significand bits, so the
 * fp32 product is exact and the single float -> fp16 round-to-nearest-even
 * below gives the same bits as an fp16 multiply.
 *
 * The fp16 <-> fp32 conversions are written here from the IEEE 754 binary16
 * definition (1 sign, 5 exponent bits with bias 15, 10 fraction bits).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bits_to_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float oracle_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t frac = h & 0x3FF;
  if (exp == 0x1F) return bits_to_float(sign | 0x7F800000u | (frac << 13));  /* inf / nan */
  if (exp == 0) {
    /* zero or subnormal: value = frac * 2^-24, exact in fp32 */
    float v = (float)frac * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  return bits_to_float(sign | ((exp - 15 + 127) << 23) | (frac << 13));
}

uint16_t oracle_float_to_half(float f) {
  uint32_t u = float_to_bits(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000);
  uint32_t a = u & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) {                      /* inf or nan */
    if (a == 0x7F800000u) return sign | 0x7C00;
    return sign | 0x7E00 | (uint16_t)((a >> 13) & 0x3FF);
  }
  int32_t e = (int32_t)(a >> 23) - 127;        /* unbiased exponent */
  uint32_t m = (a & 0x7FFFFF) | 0x800000;      /* 24-bit significand */
  if (e > 15) return sign | 0x7C00;            /* overflow -> inf */
  if (e >= -14) {                              /* normal half */
    uint32_t half_m = m >> 13;                 /* 11 bits incl. hidden one */
    uint32_t rem = m & 0x1FFF;
    uint32_t he = (uint32_t)(e + 15);
    uint32_t r = (he << 10) + (half_m - 0x400);
    if (rem > 0x1000 || (rem == 0x1000 && (half_m & 1))) r += 1;  /* RNE; carry may bump exp */
    if (r >= 0x7C00) return sign | 0x7C00;
    return sign | (uint16_t)r;
  }
  /* subnormal half: value = q * 2^-24 with q = m * 2^(e - 23 + 24) */
  if (a == 0) return sign;
  int32_t shift = -e - 14 + 13;                /* bits dropped from the 24-bit significand */
  if (shift > 24) return sign;                 /* below half of the smallest subnormal */
  uint32_t q = m >> shift;
  uint32_t rem = m & ((1u << shift) - 1);
  uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (q & 1))) q += 1;
  return sign | (uint16_t)q;                   /* q == 0x400 rolls into the smallest normal */
}

/* shift of element e (0..7) inside a packed word: kernels/awq_gemm.py:38 */
static int awq_shift(int e) { return ((e / 2) + (e % 2) * 4) * 4; }

/*
 * Dequantize packed AWQ weights to fp16 bits.
 *   qweight int32 [K, N/8], qzeros int32 [K/gs, N/8], scales fp16 [K/gs, N]
 *   out fp16 [K, N]
 * Mirrors _dequant_awq_kernel (kernels/awq_gemm.py:14-63).  Returns 0, or -1 on
 * a bad shape.
 */
int oracle_awq_dequant(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                       uint16_t* out, int64_t K, int64_t N, int64_t group_size) {
  if (K <= 0 || N <= 0 || (N % 8) || group_size <= 0 || (K % group_size)) return -1;
  int64_t pn = N / 8;
  for (int64_t k = 0; k < K; ++k) {
    int64_t g = k / group_size;
    for (int64_t n = 0; n < N; ++n) {
      int e = (int)(n % 8);
      uint32_t qw = (uint32_t)qweight[k * pn + n / 8];
      uint32_t qz = (uint32_t)qzeros[g * pn + n / 8];
      int w = (int)((qw >> awq_shift(e)) & 0xF);
      int z = (int)((qz >> awq_shift(e)) & 0xF);
      float s = oracle_half_to_float(scales[g * N + n]);
      out[k * N + n] = oracle_float_to_half((float)(w - z) * s);
    }
  }
  return 0;
}

/*
 * out[M, N] (fp32) = x[M, K] (fp16 bits) @ dequant(W)[K, N], fp32 accumulation
 * in k order.  This is the reference's dequantize-then-matmul path
 * (test/compare_benchmark.py:72-95, inference/baseline_kernels.py:36-60) with the
 * matmul carried out in fp32 on the host.
 */
int oracle_awq_gemm_f32(const uint16_t* x, int64_t M, const int32_t* qweight, const int32_t* qzeros,
                        const uint16_t* scales, int64_t K, int64_t N, int64_t group_size, float* out,
                        uint16_t* w_scratch /* K*N fp16, caller-owned */) {
  if (M <= 0) return -1;
  int rc = oracle_awq_dequant(qweight, qzeros, scales, w_scratch, K, N, group_size);
  if (rc) return rc;
  for (int64_t i = 0; i < M * N; ++i) out[i] = 0.0f;
  for (int64_t m = 0; m < M; ++m) {
    float* o = out + m * N;
    for (int64_t k = 0; k < K; ++k) {
      float xv = oracle_half_to_float(x[m * K + k]);
      const uint16_t* wr = w_scratch + k * N;
      for (int64_t n = 0; n < N; ++n) o[n] += xv * oracle_half_to_float(wr[n]);
    }
  }
  return 0;
}

/* Exported for tests that check the conversions on their own. */
void oracle_float_to_half_array(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_float_to_half(in[i]);
}
