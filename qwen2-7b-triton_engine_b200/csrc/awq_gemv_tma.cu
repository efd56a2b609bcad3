// awq_gemv_tma.cu -- decode AWQ W4A16 product (M <= 16 per token chunk), TMA-streamed,
// cluster-reduced.  The fast path of the decode branch; awq_gemv.cu keeps the generic
// kernel for shapes TMA cannot describe (N % 32 != 0, unaligned pointers).
//
// Replaces the M <= 4 dequant + torch.matmul branch of awq_gemm_forward
// (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:251-266) and small-M calls
// of _awq_gemm_kernel (kernels/awq_gemm.py:152-228).
//
// Data movement
//   * every warp owns a ring of kStages shared-memory stages; stage = one "block"
//     of 8 K-rows x 32 packed words (1 KB) of the CTA's 256-column strip, fetched
//     with one 2-D TMA load (128-byte swizzle) and completed on the stage mbarrier.
//     Bytes in flight are set by the ring depth, not by registers or occupancy.
//   * lane (g = lane/4, t = lane%4) reads rows t and t+4 of a stage as 16 bytes
//     from word chunk c(g) = (g >> 1) | ((g & 1) << 2); with the swizzle
//     (chunk ^ row) the 8 lanes of each shared-memory phase hit 8 distinct
//     16-byte bank groups.
//   * the CTA's activations are staged once (16-byte vector loads) as xs[m][k].
// Math (same as awq_gemv.cu): dequantized pairs feed mma.sync.m16n8k16 with the
//   activations spread over the (token, pair-slot) B columns; for M <= 4 the exact
//   integer (w - z) * x sums of a group are scaled in fp32 at the group's end, for
//   M > 4 W is rounded to fp16 first exactly as the reference does.
// Split-K: the CS CTAs of a thread-block cluster split K for one strip; each reduces
//   its 8 warps in shared memory, then after a cluster barrier CTA r sums column slice
//   r of all CS partials through distributed shared memory (fixed rank order, so the
//   result is deterministic) and writes fp16.  No global workspace, no atomics.
// Every mbarrier wait is bounded (status word + early exit); both cluster barriers
// are reached by every thread on every path, so a time-out never strands a peer CTA.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "awq_common.cuh"
#include "awq_internal.h"
#include "awq_sm100.cuh"

namespace awq {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 8;                 // per-warp ring depth (1 KB stages)
constexpr int kStripN = 256;
constexpr uint32_t kStageBytes = 1024;
constexpr uint32_t kRingBytes = kWarps * kStages * kStageBytes;   // 64 KB
constexpr int kRedStride = 264;

struct TmaGemvArgs {
  const __half* x;
  int64_t ldx;
  const int32_t* qz;
  const __half* scales;
  __half* out;
  int64_t ldo;
  int M, N, K, gs, PN, KB;
  int cs;          // CTAs per cluster (split-K factor)
  int bps;         // 8-row blocks per CTA
  int xs_stride;   // halves per token row of xs
  int* status;
};

__device__ __forceinline__ void mma_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int TOKSETS>
__global__ void __launch_bounds__(kThreads, 1)
gemv_tma_kernel(const __grid_constant__ CUtensorMap tmW, const TmaGemvArgs a) {
  constexpr int MP = 4 * TOKSETS;
  constexpr bool SPOST = (TOKSETS == 1);
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;
  unsigned char* sgen = smem_raw + (sbase - base_raw);
  // layout: ring | red (MP x 264 fp32) | bars (kWarps x kStages) | xs
  const uint32_t off_red = kRingBytes;
  const uint32_t off_bar = off_red + MP * kRedStride * 4;
  const uint32_t off_xs = off_bar + kWarps * kStages * 8;
  float* red = reinterpret_cast<float*>(sgen + off_red);
  __half* xs = reinterpret_cast<__half*>(sgen + off_xs);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rank = (int)cluster_ctarank();          // == blockIdx.x (cluster spans x)
  const int strip = blockIdx.y;
  const int zc = blockIdx.z;
  const int m0 = zc * 16;
  const int Mc = min(MP, a.M - m0);
  const int cb0 = rank * a.bps;
  const int cb1 = min(a.KB, cb0 + a.bps);
  const int nb = max(0, cb1 - cb0);
  const int per = (nb + kWarps - 1) / kWarps;
  const int b0 = cb0 + min(nb, warp * per);
  const int b1 = cb0 + min(nb, (warp + 1) * per);
  const int nblk = b1 - b0;
  const int krow0 = cb0 * 8;
  const int Kc = nb * 8;

  const uint32_t ring = sbase + (uint32_t)warp * kStages * kStageBytes;
  const uint32_t bars = sbase + off_bar + (uint32_t)warp * kStages * 8;

  // ---- barriers, then start streaming before anything else -------------------------
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) sm100::mbar_init(bars + 8 * s, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmW);
  }
  __syncwarp();
  if (lane == 0) {
    for (int i = 0; i < kStages && i < nblk; ++i) {
      sm100::mbar_arrive_expect_tx(bars + 8 * i, kStageBytes);
      sm100::tma_load_2d(ring + i * kStageBytes, &tmW, bars + 8 * i, strip * 32, (b0 + i) * 8);
    }
  }

  // ---- stage activations xs[m][k] (zeros for tokens >= Mc) -------------------------
  {
    const int vecs = Kc / 8;                         // 16-byte vectors per token row
    for (int i = tid; i < MP * vecs; i += kThreads) {
      const int m = i / vecs, v = i - m * vecs;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (m < Mc)
        val = __ldg(reinterpret_cast<const uint4*>(a.x + (int64_t)(m0 + m) * a.ldx + krow0) + v);
      *reinterpret_cast<uint4*>(xs + m * a.xs_stride + v * 8) = val;
    }
  }
  __syncthreads();

  const int chunk = (g >> 1) | ((g & 1) << 2);       // conflict-free word chunk
  const int wc0 = strip * 32 + chunk * 4;            // first packed word of this lane
  float acc[TOKSETS][8][4];
#pragma unroll
  for (int s = 0; s < TOKSETS; ++s)
#pragma unroll
    for (int q = 0; q < 8; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][q][i] = 0.f;
  float pacc[SPOST ? 8 : 1][4];
#pragma unroll
  for (int q = 0; q < (SPOST ? 8 : 1); ++q)
#pragma unroll
    for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;

  uint32_t zcst[4][4], scl[4][4];
  int grp_end = -1;
  // raw zeros / scales of the next group, loaded one group ahead
  uint4 pf_z = make_uint4(0, 0, 0, 0), pf_s[4];
  int pf_grp = -1;
  auto load_group = [&](int grp) {
    pf_grp = grp;
    pf_z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int c = 0; c < 4; ++c) pf_s[c] = make_uint4(0, 0, 0, 0);
    if (wc0 < a.PN) {
      pf_z = __ldg(reinterpret_cast<const uint4*>(a.qz + (int64_t)grp * a.PN + wc0));
#pragma unroll
      for (int c = 0; c < 4; ++c)
        pf_s[c] = __ldg(reinterpret_cast<const uint4*>(a.scales + (int64_t)grp * a.N + (wc0 + c) * 8));
    }
  };
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

  int i_fail = nblk;                    // first block whose stage never arrived
  for (int i = 0; i < nblk; ++i) {
    const int s = i % kStages;
    if (!sm100::mbar_wait_bounded(bars + 8 * s, (i / kStages) & 1, a.status)) {
      i_fail = i;
      break;
    }
    const uint32_t st = ring + s * kStageBytes;
    const uint4 va = lds128(st + t * 128 + ((uint32_t)(chunk ^ t) << 4));
    const uint4 vb = lds128(st + (t + 4) * 128 + ((uint32_t)(chunk ^ (t + 4)) << 4));
    const int bb = b0 + i;
    const int k0 = bb * 8;
    if (k0 >= grp_end) {
      if (grp_end >= 0) flush();
      const int grp = k0 / a.gs;
      if (grp != pf_grp) load_group(grp);           // first group of the warp's range
      grp_end = (grp + 1) * a.gs;
      const uint32_t zw[4] = {pf_z.x, pf_z.y, pf_z.z, pf_z.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        zero_consts(zw[c], zcst[c]);
        scl[c][0] = pf_s[c].x; scl[c][1] = pf_s[c].y; scl[c][2] = pf_s[c].z; scl[c][3] = pf_s[c].w;
      }
      // fetch the next group now; it has a whole group of blocks to arrive
      if (grp_end < b1 * 8) load_group(grp + 1);
    }
    uint32_t bf0[TOKSETS], bf1[TOKSETS];
    const int kl = k0 - krow0;
#pragma unroll
    for (int s2 = 0; s2 < TOKSETS; ++s2) {
      const int m = 4 * s2 + (g >> 1);
      const uint32_t xa = __half_as_ushort(xs[m * a.xs_stride + kl + t]);
      const uint32_t xb = __half_as_ushort(xs[m * a.xs_stride + kl + t + 4]);
      bf0[s2] = (g & 1) ? (xa << 16) : xa;
      bf1[s2] = (g & 1) ? (xb << 16) : xb;
    }
    const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
    const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t da[4], db[4];
      if constexpr (SPOST) {
        unpack_minus_zero(wa[c], zcst[c], da);
        unpack_minus_zero(wb[c], zcst[c], db);
      } else {
        dequant_word(wa[c], zcst[c], scl[c], da);
        dequant_word(wb[c], zcst[c], scl[c], db);
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int q = 2 * c + jj;
        if constexpr (SPOST) {
          mma_16816(pacc[q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf0[0], bf1[0]);
        } else {
#pragma unroll
          for (int s2 = 0; s2 < TOKSETS; ++s2)
            mma_16816(acc[s2][q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf0[s2],
                      bf1[s2]);
        }
      }
    }
    // refill this stage with block i + kStages: every lane's reads of it have
    // completed (their values were consumed above), so the copy may overwrite it
    __syncwarp();
    if (lane == 0 && i + kStages < nblk) {
      sm100::mbar_arrive_expect_tx(bars + 8 * s, kStageBytes);
      sm100::tma_load_2d(st, &tmW, bars + 8 * s, strip * 32, (b0 + i + kStages) * 8);
    }
  }
  if (grp_end >= 0) flush();
  if (i_fail < nblk && lane == 0) {
    // a stage never arrived: wait (bounded) for the copies this warp still has in
    // flight -- blocks [i_fail, i_fail + kStages) -- before the CTA may exit
    for (int i = i_fail; i < nblk && i < i_fail + kStages; ++i)
      sm100::mbar_wait_bounded(bars + 8 * (i % kStages), (i / kStages) & 1, nullptr, 50000000ull);
  }
  __syncwarp();

  // ---- CTA reduction: warps add into red[m][n] in fixed order ----------------------
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int s2 = 0; s2 < TOKSETS; ++s2) {
        const int m = 4 * s2 + t;
        if (m < MP) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4* dst = reinterpret_cast<float4*>(red + m * kRedStride + 32 * chunk + 4 * q);
            if (w == 0) {
              *dst = make_float4(acc[s2][q][0], acc[s2][q][1], acc[s2][q][2], acc[s2][q][3]);
            } else {
              float4 v = *dst;
              v.x += acc[s2][q][0]; v.y += acc[s2][q][1]; v.z += acc[s2][q][2]; v.w += acc[s2][q][3];
              *dst = v;
            }
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- cluster reduction over distributed shared memory ----------------------------
  cluster_sync_all();                                  // every CTA's red is complete
  const int cw = kStripN / a.cs;                       // columns reduced by this CTA
  const int nbase = strip * kStripN;
  const uint32_t red_addr = sbase + off_red;
  for (int idx = tid; idx < Mc * cw; idx += kThreads) {
    const int m = idx / cw;
    const int nl = rank * cw + (idx - m * cw);
    const uint32_t la = red_addr + (uint32_t)(m * kRedStride + nl) * 4u;
    float v = 0.f;
    for (int r = 0; r < a.cs; ++r) v += ld_dsmem_f32(la, (uint32_t)r);
    const int n = nbase + nl;
    if (n < a.N) a.out[(int64_t)(m0 + m) * a.ldo + n] = __float2half_rn(v);
  }
  cluster_sync_all();                                  // keep smem alive for the readers
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

template <int TOKSETS>
size_t smem_bytes(int xs_stride) {
  const int MP = 4 * TOKSETS;
  return 1024 + kRingBytes + (size_t)MP * kRedStride * 4 + kWarps * kStages * 8 +
         (size_t)MP * xs_stride * 2;
}

template <int TOKSETS>
cudaError_t launch_t(const CUtensorMap& tm, const TmaGemvArgs& a, int strips, int zchunks,
                     size_t smem, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(gemv_tma_kernel<TOKSETS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (attr == cudaSuccess)
      attr = cudaFuncSetAttribute(gemv_tma_kernel<TOKSETS>,
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
  if (attr != cudaSuccess) return attr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cs, strips, zchunks);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.cs;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<TOKSETS>, tm, a);
}

}  // namespace

bool gemv_tma_supported(const int32_t* qweight, int64_t N, int64_t ldx, const void* x) {
  return (N % 32 == 0) && ((reinterpret_cast<uintptr_t>(qweight) & 15) == 0) &&
         ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 8 == 0) && encode_fn() != nullptr;
}

int gemv_tma_cluster_size(int64_t M, int64_t N, int64_t K, int num_sms, int max_cs) {
  const int64_t strips = (N + kStripN - 1) / kStripN;
  const int64_t zchunks = (M + 15) / 16;
  const int64_t KB = K / 8;
  int cs = 1;
  while (cs < max_cs && strips * zchunks * cs * 2 <= (int64_t)num_sms * 2 && KB / (cs * 2) >= 16)
    cs *= 2;
  return cs;
}

cudaError_t launch_gemv_tma(const void* x, int64_t ldx, const int32_t* qweight,
                            const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                            int M, int N, int K, int group_size, int num_sms, int max_cs,
                            int* dev_status, cudaStream_t stream) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)(N / 8), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)N / 2};
  cuuint32_t box[2] = {32, 8};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const int strips = (N + kStripN - 1) / kStripN;
  const int cs = gemv_tma_cluster_size(M < 16 ? M : 16, N, K, num_sms, max_cs);
  TmaGemvArgs a;
  a.ldx = ldx;
  a.qz = qzeros;
  a.scales = static_cast<const __half*>(scales);
  a.ldo = ldo;
  a.N = N; a.K = K; a.gs = group_size; a.PN = N / 8; a.KB = K / 8;
  a.cs = cs;
  a.bps = (a.KB + cs - 1) / cs;
  a.xs_stride = a.bps * 8 + 8;                        // +16 B staggers token rows
  a.status = dev_status;
  const int64_t mtot = M;
  const int mc = M < 16 ? M : 16;
  const int toksets = mc <= 4 ? 1 : (mc <= 8 ? 2 : 4);
  const int max_z = 65535;
  for (int64_t m0 = 0; m0 < mtot; m0 += (int64_t)max_z * 16) {
    const int64_t rows = (mtot - m0 < (int64_t)max_z * 16) ? (mtot - m0) : (int64_t)max_z * 16;
    a.x = static_cast<const __half*>(x) + m0 * ldx;
    a.out = static_cast<__half*>(out) + m0 * ldo;
    a.M = (int)rows;
    const int z = (int)((rows + 15) / 16);
    cudaError_t e;
    switch (toksets) {
      case 1: e = launch_t<1>(tm, a, strips, z, smem_bytes<1>(a.xs_stride), stream); break;
      case 2: e = launch_t<2>(tm, a, strips, z, smem_bytes<2>(a.xs_stride), stream); break;
      default: e = launch_t<4>(tm, a, strips, z, smem_bytes<4>(a.xs_stride), stream); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t gemv_tma_smem_bytes(int64_t M, int64_t N, int64_t K, int num_sms, int max_cs) {
  const int cs = gemv_tma_cluster_size(M < 16 ? M : 16, N, K, num_sms, max_cs);
  const int bps = (int)((K / 8 + cs - 1) / cs);
  const int mc = M < 16 ? (int)M : 16;
  const int xs_stride = bps * 8 + 8;
  return mc <= 4 ? smem_bytes<1>(xs_stride) : (mc <= 8 ? smem_bytes<2>(xs_stride) : smem_bytes<4>(xs_stride));
}

}  // namespace awq
