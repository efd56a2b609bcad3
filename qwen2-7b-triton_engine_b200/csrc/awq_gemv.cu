// awq_gemv.cu -- decode / skinny AWQ W4A16 product (M <= 16 per token chunk) on sm_100a.
//
// Replaces the M <= 4 branch of awq_gemm_forward (dequant to a global fp16 buffer,
// then torch.matmul; songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:251-266) and
// the small-M use of _awq_gemm_kernel (kernels/awq_gemm.py:152-228).  Weights are read
// once, straight from the packed layout, at 0.52 B per weight instead of ~4.5 B.
//
// Work decomposition
//   strip  : 256 output columns = 32 packed words; one warp covers a strip, lane
//            (g = lane/4, t = lane%4) holds the 4 words [4g, 4g+4) of the strip
//   block  : 8 rows of K; per block a thread loads rows k0+t and k0+t+4 with one
//            16-byte load each (a warp reads 8 full 128-byte lines)
//   CTA    : 4 warps on one strip and one contiguous range of blocks (a "split");
//            the warps split the range and reduce their partials in shared memory
//   grid   : (strips, splits, token chunks of 16); splits > 1 adds a split-K
//            reduction through an fp32 workspace in which the last CTA of a strip
//            (arrival counter) sums the partials in split order -- deterministic.
//
// Math: dequantized pairs go straight from registers into mma.sync.m16n8k16
// (fp16 x fp16 -> fp32).  The weight tile is the A operand: row r of the MMA is
// one element pair (2j, 2j+1) of one packed word, and the 16 A columns are 8 rows
// of K times 2 pair slots.  The activation is "spread" over the 8 B columns as
// (token, slot): B[2i+p][2m+q] = x[m][k0+i] if p == q else 0, so C[r][2m+q] is the
// dot product for element 2j+q of row r and token m.  No register transposes
// are needed, and 4 tokens share one MMA.  Products accumulate in fp32.
//   M <= 4 per chunk: the MMAs accumulate the exact integers (w - z) times x over
//     one group and the fp32 scale is applied once per group (no per-weight fp16
//     multiply; the result is at least as accurate as the reference's).
//   M  > 4: W is formed exactly as the reference forms it (fp16 (w - z) * scale)
//     before the MMA.
#include "awq_common.cuh"
#include "awq_internal.h"

namespace awq {

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kStripN = 256;
constexpr int kPrefetch = 4;     // blocks of 8 rows in flight per warp
constexpr int kRedStride = 264;  // padded row of the cross-warp reduction buffer
// Split-K arrival counters live in a fixed region at the head of the workspace
// (kCounterRegionBytes, awq_internal.h), so a call's fp32 partials (which follow the
// region) can never land on another call's counters.

__device__ __forceinline__ void mma_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct GemvArgs {
  const __half* x;
  int64_t ldx;
  const int32_t* qw;
  const int32_t* qz;
  const __half* scales;
  __half* out;
  int64_t ldo;
  int M, N, K, gs, PN;
  int strips, splits, bps;
  float* ws;        // [zchunks][splits][16][strips*256]
  int* counters;    // [zchunks][strips]
  const __half* bias;   // fp16 [N] added to every output row in fp32, or null
};

// Output element: the fp32 sum plus the column's bias (when given), rounded once.
__device__ __forceinline__ __half out_value(const GemvArgs& a, int n, float v) {
  if (a.bias) v += __half2float(a.bias[n]);
  return __float2half_rn(v);
}

template <bool VEC>
__device__ __forceinline__ void load_words(const GemvArgs& a, int row, int wc0, uint32_t w[4]) {
  const int32_t* p = a.qw + (int64_t)row * a.PN + wc0;
  if constexpr (VEC) {
    // PN % 4 == 0 here, so the 4 words of a lane are all in range or all past the end
    if (wc0 < a.PN) {
      uint4 v = ldg_stream_v4(p);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else {
      w[0] = w[1] = w[2] = w[3] = 0u;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) w[c] = (wc0 + c < a.PN) ? ldg_stream_u32(p + c) : 0u;
  }
}

template <int TOKSETS, bool VEC>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
  constexpr int MP = 4 * TOKSETS;          // padded tokens held by a CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* xs = reinterpret_cast<__half*>(smem_raw);   // [rows of the split][MP]
  float* red = reinterpret_cast<float*>(smem_raw);    // reused after the main loop
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int strip = blockIdx.x, split = blockIdx.y, zc = blockIdx.z;
  const int m0 = zc * 16;
  const int Mc = min(MP, a.M - m0);
  const int KB = a.K >> 3;
  const int cb0 = split * a.bps;
  const int cb1 = min(KB, cb0 + a.bps);
  const int nb = cb1 - cb0;
  const int per = (nb + kGemvWarps - 1) / kGemvWarps;
  const int b0 = cb0 + min(nb, warp * per);
  const int b1 = cb0 + min(nb, (warp + 1) * per);
  const int krow0 = cb0 * 8;

  // ---- stage this split's activations: xs[k][m] (zero for tokens >= Mc) -------------
  for (int i = tid; i < nb * 8 * MP; i += kGemvThreads) {
    const int m = i / (nb * 8);
    const int kk = i - m * (nb * 8);
    __half v = __float2half_rn(0.f);
    if (m < Mc) v = a.x[(int64_t)(m0 + m) * a.ldx + krow0 + kk];
    xs[kk * MP + m] = v;
  }
  __syncthreads();

  const int wc0 = strip * 32 + g * 4;      // first packed word of this lane
  float acc[TOKSETS][8][4];
#pragma unroll
  for (int s = 0; s < TOKSETS; ++s)
#pragma unroll
    for (int q = 0; q < 8; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][q][i] = 0.f;

  uint32_t wa[kPrefetch][4], wb[kPrefetch][4];
#pragma unroll
  for (int i = 0; i < kPrefetch; ++i) {
    if (b0 + i < b1) {
      load_words<VEC>(a, (b0 + i) * 8 + t, wc0, wa[i]);
      load_words<VEC>(a, (b0 + i) * 8 + t + 4, wc0, wb[i]);
    }
  }

  // SPOST (one 4-token set): the MMAs accumulate exact (w - z) * x per group into
  // pacc and the fp32 scale is applied when the group ends, which saves the fp16
  // scale multiply per weight.  Otherwise W is rounded to fp16 first, exactly like
  // the reference's dequantized matrix.
  constexpr bool SPOST = (TOKSETS == 1);
  float pacc[SPOST ? 8 : 1][4];
#pragma unroll
  for (int q = 0; q < (SPOST ? 8 : 1); ++q)
#pragma unroll
    for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;

  uint32_t zcst[4][4], scl[4][4];
  int grp_end = -1;                 // first K row past the current group
  const int64_t N = a.N;

  auto flush = [&]() {
    if constexpr (SPOST) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = q >> 1, jj = q & 1;
        const float2 sa = __half22float2(u32_as_h2(scl[c][2 * jj]));
        const float2 sb = __half22float2(u32_as_h2(scl[c][2 * jj + 1]));
        acc[0][q][0] = fmaf(sa.x, pacc[q][0], acc[0][q][0]);
        acc[0][q][1] = fmaf(sa.y, pacc[q][1], acc[0][q][1]);
        acc[0][q][2] = fmaf(sb.x, pacc[q][2], acc[0][q][2]);
        acc[0][q][3] = fmaf(sb.y, pacc[q][3], acc[0][q][3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;
      }
    }
  };

  for (int b = b0; b < b1; b += kPrefetch) {
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i) {
      const int bb = b + i;
      if (bb < b1) {
        const int k0 = bb * 8;
        if (k0 >= grp_end) {
          if (grp_end >= 0) flush();
          const int grp = k0 / a.gs;
          grp_end = (grp + 1) * a.gs;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int wc = wc0 + c;
            uint32_t zw = 0;
            uint4 s4 = make_uint4(0, 0, 0, 0);
            if (wc < a.PN) {
              zw = static_cast<uint32_t>(__ldg(a.qz + (int64_t)grp * a.PN + wc));
              s4 = __ldg(reinterpret_cast<const uint4*>(a.scales + (int64_t)grp * N + wc * 8));
            }
            zero_consts(zw, zcst[c]);
            scl[c][0] = s4.x; scl[c][1] = s4.y; scl[c][2] = s4.z; scl[c][3] = s4.w;
          }
        }
        // B fragments (spread activations), one pair per 4-token set
        uint32_t bf0[TOKSETS], bf1[TOKSETS];
        const int kl = k0 - krow0;
#pragma unroll
        for (int s = 0; s < TOKSETS; ++s) {
          const int m = 4 * s + (g >> 1);
          const uint32_t xa = __half_as_ushort(xs[(kl + t) * MP + m]);
          const uint32_t xb = __half_as_ushort(xs[(kl + t + 4) * MP + m]);
          bf0[s] = (g & 1) ? (xa << 16) : xa;
          bf1[s] = (g & 1) ? (xb << 16) : xb;
        }
        // dequantize the 8 words, feed 8 MMA tiles per token set
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t da[4], db[4];
          if constexpr (SPOST) {
            unpack_minus_zero(wa[i][c], zcst[c], da);
            unpack_minus_zero(wb[i][c], zcst[c], db);
          } else {
            dequant_word(wa[i][c], zcst[c], scl[c], da);
            dequant_word(wb[i][c], zcst[c], scl[c], db);
          }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int q = 2 * c + jj;
            if constexpr (SPOST) {
              mma_16816(pacc[q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf0[0],
                        bf1[0]);
            } else {
#pragma unroll
              for (int s = 0; s < TOKSETS; ++s)
                mma_16816(acc[s][q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1],
                          bf0[s], bf1[s]);
            }
          }
        }
        const int nx = bb + kPrefetch;
        if (nx < b1) {
          load_words<VEC>(a, nx * 8 + t, wc0, wa[i]);
          load_words<VEC>(a, nx * 8 + t + 4, wc0, wb[i]);
        }
      }
    }
  }
  if (grp_end >= 0) flush();

  // ---- cross-warp reduction in shared memory (fixed order: warp 0, 1, 2, 3) --------
  __syncthreads();                                  // xs is dead; reuse as red
  for (int w = 0; w < kGemvWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int s = 0; s < TOKSETS; ++s) {
        const int m = 4 * s + t;
        if (m < Mc) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4* dst = reinterpret_cast<float4*>(red + m * kRedStride + 32 * g + 4 * q);
            if (w == 0) {
              *dst = make_float4(acc[s][q][0], acc[s][q][1], acc[s][q][2], acc[s][q][3]);
            } else {
              float4 v = *dst;
              v.x += acc[s][q][0]; v.y += acc[s][q][1]; v.z += acc[s][q][2]; v.w += acc[s][q][3];
              *dst = v;
            }
          }
        }
      }
    }
    __syncthreads();
  }

  const int NP = a.strips * kStripN;
  const int nbase = strip * kStripN;
  if (a.splits == 1) {
    for (int idx = tid; idx < Mc * kStripN; idx += kGemvThreads) {
      const int m = idx / kStripN, nl = idx - m * kStripN;
      const int n = nbase + nl;
      if (n < a.N) a.out[(int64_t)(m0 + m) * a.ldo + n] = out_value(a, n, red[m * kRedStride + nl]);
    }
    return;
  }

  float* part = a.ws + ((int64_t)zc * a.splits + split) * 16 * NP;
  for (int idx = tid; idx < Mc * kStripN; idx += kGemvThreads) {
    const int m = idx / kStripN, nl = idx - m * kStripN;
    __stcg(part + (int64_t)m * NP + nbase + nl, red[m * kRedStride + nl]);
  }
  __threadfence();
  __syncthreads();
  int* ctr = a.counters + zc * a.strips + strip;
  if (tid == 0) s_last = (atomicAdd(ctr, 1) == a.splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* base = a.ws + (int64_t)zc * a.splits * 16 * NP;
  for (int idx = tid; idx < Mc * kStripN; idx += kGemvThreads) {
    const int m = idx / kStripN, nl = idx - m * kStripN;
    const int n = nbase + nl;
    float v = 0.f;
    for (int sp = 0; sp < a.splits; ++sp) v += __ldcg(base + ((int64_t)sp * 16 + m) * NP + n);
    if (n < a.N) a.out[(int64_t)(m0 + m) * a.ldo + n] = out_value(a, n, v);
  }
  if (tid == 0) *ctr = 0;                           // leave the counter at zero for the next call
}

// ----------------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------------
static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool plan_gemv(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms, bool vec_ok,
               GemvPlan* plan) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 8 || K % 8 || group_size <= 0 || group_size % 8 ||
      K % group_size)
    return false;
  GemvPlan p{};
  p.strips = (int)((N + kStripN - 1) / kStripN);
  if (p.strips > kMaxCounters) return false;
  // token chunks of 16 per launch, bounded so that one launch's counters fit the
  // fixed counter region; larger M is covered by several launches in stream order
  const int64_t chunks = (M + 15) / 16;
  const int64_t max_chunks = kMaxCounters / p.strips;
  p.zchunks = (int)(chunks < max_chunks ? chunks : max_chunks);
  const int64_t mc = M < 16 ? M : 16;
  p.toksets = mc <= 4 ? 1 : (mc <= 8 ? 2 : 4);
  p.vec = vec_ok ? 1 : 0;
  const int64_t KB = K / 8;
  const int64_t target = (int64_t)num_sms * 4;                 // 4 CTAs of 4 warps per SM
  int64_t splits = (target + (int64_t)p.strips * p.zchunks - 1) / ((int64_t)p.strips * p.zchunks);
  const int64_t max_splits = (KB + 7) / 8;                     // >= 8 blocks per CTA
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  const int MP = 4 * p.toksets;
  for (;;) {
    int64_t bps = (KB + splits - 1) / splits;
    splits = (KB + bps - 1) / bps;
    size_t xs_bytes = (size_t)bps * 8 * MP * sizeof(uint16_t);
    size_t red_bytes = (size_t)MP * kRedStride * sizeof(float);
    size_t smem = xs_bytes > red_bytes ? xs_bytes : red_bytes;
    if (smem <= 48 * 1024 || splits >= KB) {
      p.bps = (int)bps;
      p.splits = (int)splits;
      p.smem = smem;
      break;
    }
    splits *= 2;
  }
  if (p.smem > 48 * 1024) return false;
  const size_t NP = (size_t)p.strips * kStripN;
  p.ws_partials_bytes = p.splits > 1 ? (size_t)p.zchunks * p.splits * 16 * NP * sizeof(float) : 0;
  p.ws_counter_bytes = kCounterRegionBytes;
  *plan = p;
  return true;
}

bool plan_gemv_bounded(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                       bool vec_ok, size_t max_workspace, GemvPlan* plan) {
  GemvPlan p;
  if (!plan_gemv(M, N, K, group_size, num_sms, vec_ok, &p)) return false;
  // fewer splits -> smaller partial buffer; the shared-memory bound sets the floor
  const int64_t KB = K / 8;
  const int MP = 4 * p.toksets;
  const size_t NP = (size_t)p.strips * kStripN;
  int64_t splits = p.splits;
  for (;;) {
    int64_t bps = (KB + splits - 1) / splits;
    int64_t sp = (KB + bps - 1) / bps;
    size_t xs_bytes = (size_t)bps * 8 * MP * sizeof(uint16_t);
    size_t red_bytes = (size_t)MP * kRedStride * sizeof(float);
    size_t smem = xs_bytes > red_bytes ? xs_bytes : red_bytes;
    size_t partials = sp > 1 ? (size_t)p.zchunks * sp * 16 * NP * sizeof(float) : 0;
    size_t need = sp > 1 ? kCounterRegionBytes + align_up(partials, 256) : 0;
    if (smem > 48 * 1024) return false;               // cannot shrink further
    if (need <= max_workspace) {
      p.bps = (int)bps;
      p.splits = (int)sp;
      p.smem = smem;
      p.ws_partials_bytes = partials;
      break;
    }
    if (sp <= 1) return false;
    splits = sp / 2;
  }
  *plan = p;
  return true;
}

size_t gemv_workspace_bytes(const GemvPlan& plan) {
  if (plan.splits <= 1) return 0;
  return kCounterRegionBytes + align_up(plan.ws_partials_bytes, 256);
}

template <int TOKSETS>
static void launch_t(const GemvPlan& plan, const GemvArgs& args, int zchunks, cudaStream_t stream) {
  dim3 grid(plan.strips, plan.splits, zchunks);
  if (plan.vec)
    gemv_kernel<TOKSETS, true><<<grid, kGemvThreads, plan.smem, stream>>>(args);
  else
    gemv_kernel<TOKSETS, false><<<grid, kGemvThreads, plan.smem, stream>>>(args);
}

cudaError_t launch_gemv(const GemvPlan& plan, const void* x, int64_t ldx, const int32_t* qweight,
                        const int32_t* qzeros, const void* scales, void* out, int64_t ldo, int M,
                        int N, int K, int group_size, void* workspace, cudaStream_t stream,
                        const void* bias) {
  GemvArgs a;
  a.bias = static_cast<const __half*>(bias);
  a.ldx = ldx;
  a.qw = qweight;
  a.qz = qzeros;
  a.scales = static_cast<const __half*>(scales);
  a.ldo = ldo;
  a.N = N; a.K = K; a.gs = group_size; a.PN = N / 8;
  a.strips = plan.strips; a.splits = plan.splits; a.bps = plan.bps;
  a.counters = reinterpret_cast<int*>(workspace);
  a.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegionBytes);
  // one launch per group of plan.zchunks token chunks (16 tokens each)
  const int64_t rows_per_launch = (int64_t)plan.zchunks * 16;
  for (int64_t m0 = 0; m0 < M; m0 += rows_per_launch) {
    const int64_t mrows = (M - m0 < rows_per_launch) ? (M - m0) : rows_per_launch;
    a.x = static_cast<const __half*>(x) + m0 * ldx;
    a.out = static_cast<__half*>(out) + m0 * ldo;
    a.M = (int)mrows;
    const int z = (int)((mrows + 15) / 16);
    switch (plan.toksets) {
      case 1: launch_t<1>(plan, a, z, stream); break;
      case 2: launch_t<2>(plan, a, z, stream); break;
      default: launch_t<4>(plan, a, z, stream); break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace awq
