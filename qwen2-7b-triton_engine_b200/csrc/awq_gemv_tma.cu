// awq_gemv_tma.cu -- decode AWQ W4A16 product (M <= 16 per token chunk), TMA-streamed,
// cluster-reduced.  The fast path of the decode branch; awq_gemv.cu keeps the generic
// kernel for shapes TMA cannot describe (N % 32 != 0, group_size % 32 != 0, unaligned).
//
// Replaces the M <= 4 dequant + torch.matmul branch of awq_gemm_forward
// (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:251-266) and small-M calls
// of _awq_gemm_kernel (kernels/awq_gemm.py:152-228).
//
// Roles (one CTA = 8 warps, one CTA per SM)
//   every warp owns a contiguous, stage-aligned range of the CTA's K rows and a ring of
//   shared-memory stages it refills itself: one 2-D TMA load of 32 K-rows x 32 packed
//   words (4 KB, 128-byte swizzle) per stage, completing on the stage's mbarrier.  It
//   walks its range one quantization group at a time; the inner loop over the group's
//   stages is branch-free apart from the barrier wait and the refill: 4 x (2 shared
//   loads + biased unpack + 8 mma.sync) per stage.  The group's zero/scale correction
//   runs once per group, outside that loop.
//   lane (g = lane/4, t = lane%4) reads rows t and t+4 of each 8-row block as 16 bytes
//   from word chunk c(g) = (g >> 1) | ((g & 1) << 2); with the swizzle (chunk ^ row)
//   the 8 lanes of each shared-memory phase hit 8 distinct 16-byte bank groups.
// Math: dequantized pairs feed mma.sync.m16n8k16 (fp16 x fp16 -> fp32) with the
//   activations spread over the (token, pair-slot) B columns.  For M <= 4 the MMA takes
//   the exact biased values 1024 + w / 1024 + 16 w and the zero term
//   (1024 + z) * sum(x) / (1024 + 16 z) * sum(x) is removed per group in fp32 before the
//   fp32 scale (scale / 16) is applied; for M > 4 W is rounded to fp16 first exactly as
//   the reference does.
// Split-K: the CS CTAs of a thread-block cluster split K for one 256-column strip; each
//   sums its 8 warps' partials in shared memory (one barrier, fixed order), then after a
//   cluster barrier CTA r sums column slice r of all CS partials through distributed
//   shared memory (fixed rank order, so the result is deterministic) and writes fp16.
//   With CS = 1 the CTA writes its sum directly.  No global workspace, no atomics.
// Every mbarrier wait is bounded (status word + early exit); both cluster barriers are
// reached by every thread on every path, so a time-out never strands a peer CTA.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "awq_common.cuh"
#include "awq_internal.h"
#include "awq_sm100.cuh"

namespace awq {

namespace {

constexpr int kConsumers = 8;                     // warps per CTA
constexpr int kThreads = kConsumers * 32;
constexpr int kRowsPerStage = 32;                 // four 8-row blocks per TMA copy
constexpr int kBlocksPerStage = kRowsPerStage / 8;
constexpr int kStripN = 256;
constexpr uint32_t kStageBytes = kRowsPerStage * 128;                // 4 KB
constexpr int kRedStride = 264;

template <int TOKSETS>
struct DecGeo {
  static constexpr int kStages = TOKSETS == 1 ? 4 : 2;              // per-warp ring depth
  static constexpr uint32_t kRingBytes = kConsumers * kStages * kStageBytes;
  // row stride (floats) of a warp's partial sums parked in its own ring after the loop;
  // MP rows of it must fit the warp's kStages * 4 KB
  static constexpr int kPartStride = TOKSETS == 1 ? kRedStride : kStripN;
  static_assert(4 * TOKSETS * kPartStride * 4 <= kStages * (int)kStageBytes, "partials fit the ring");
};

struct TmaGemvArgs {
  const __half* x;
  int64_t ldx;
  const int32_t* qz;
  const __half* scales;
  __half* out;
  int64_t ldo;
  int M, N, K, gs, PN, KB;
  int cs;          // CTAs per cluster (split-K factor)
  int bps;         // 8-row blocks per CTA (multiple of kBlocksPerStage)
  int xs_stride;   // halves per token row of xs
  int ngrp_cta;    // quantization groups a CTA's K range can touch (zs / ss rows)
  int l2pf;        // weight stages each warp prefetches into L2 before the dependency wait
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

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// 16-byte asynchronous global -> shared copy (no register round trip); completion is
// awaited with cp_async_wait_all.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void sts128_zero(uint32_t dst) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dst), "r"(0u) : "memory");
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

// Biased unpack: 4 half2 holding (1024 + w) for nibbles at bits 0..3 / 16..19 and
// (1024 + 16 w) for bits 4..7 / 20..23, of the word and of word >> 8 -- exact values,
// element pairs (0,1), (2,3), (4,5), (6,7).  No zero subtraction per weight.
__device__ __forceinline__ void unpack_biased(uint32_t w, uint32_t d[4]) {
  const uint32_t w8 = w >> 8;
  d[0] = lop3_and_or(w, kLoMask, kMagic);
  d[1] = lop3_and_or(w, kHiMask, kMagic);
  d[2] = lop3_and_or(w8, kLoMask, kMagic);
  d[3] = lop3_and_or(w8, kHiMask, kMagic);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Stage-aligned K range [b0, b1) (in 8-row blocks) of consumer warp w of a CTA whose
// range is [cb0, cb0 + nb).
__device__ __forceinline__ void warp_range(int cb0, int nb, int w, int& b0, int& b1) {
  int per = (nb + kConsumers - 1) / kConsumers;
  per = (per + kBlocksPerStage - 1) / kBlocksPerStage * kBlocksPerStage;
  b0 = cb0 + min(nb, w * per);
  b1 = cb0 + min(nb, (w + 1) * per);
}

template <int TOKSETS>
__global__ void __launch_bounds__(kThreads, 1)
gemv_tma_kernel(const __grid_constant__ CUtensorMap tmW, const TmaGemvArgs a) {
  constexpr int MP = 4 * TOKSETS;
  constexpr bool BIAS = (TOKSETS == 1);
  constexpr int kStages = DecGeo<TOKSETS>::kStages;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;
  unsigned char* sgen = smem_raw + (sbase - base_raw);
  // layout: ring | red (MP x 264 fp32) | stage bars | abort | xs | zs | ss
  const uint32_t off_red = DecGeo<TOKSETS>::kRingBytes;
  const uint32_t off_full = off_red + MP * kRedStride * 4;
  const uint32_t off_misc = off_full + kConsumers * kStages * 8;
  const uint32_t off_xs = off_misc + 16;
  const uint32_t off_zs = off_xs + (uint32_t)MP * a.xs_stride * 2;
  const uint32_t off_ss = off_zs + (uint32_t)a.ngrp_cta * 128;
  float* red = reinterpret_cast<float*>(sgen + off_red);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + off_misc);
  __half* xs = reinterpret_cast<__half*>(sgen + off_xs);
  uint32_t* zs = reinterpret_cast<uint32_t*>(sgen + off_zs);    // [group][32 words]
  __half* ss = reinterpret_cast<__half*>(sgen + off_ss);        // [group][256]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rank = (int)cluster_ctarank();          // == blockIdx.x (cluster spans x)
  const int strip = blockIdx.y;
  const int zc = blockIdx.z;
  const int m0 = zc * MP;                           // token chunk of this CTA
  const int Mc = min(MP, a.M - m0);
  const int cb0 = rank * a.bps;
  const int cb1 = min(a.KB, cb0 + a.bps);
  const int nb = max(0, cb1 - cb0);
  const int krow0 = cb0 * 8;
  const int Kc = nb * 8;
  auto full_bar = [&](int w, int s) { return sbase + off_full + (uint32_t)(w * kStages + s) * 8u; };
  auto stage_addr = [&](int w, int s) {
    return sbase + (uint32_t)(w * kStages + s) * kStageBytes;
  };

  // every warp initialises its own stage barriers and starts its own stream
  int b0, b1;
  warp_range(cb0, nb, warp, b0, b1);
  const int nst = (b1 - b0) / kBlocksPerStage;
  if (lane == 0) {
    for (int s2 = 0; s2 < kStages; ++s2) sm100::mbar_init(full_bar(warp, s2), 1);
    sm100::fence_mbar_init();
    if (warp == 0) {
      *abort_flag = 0;
      sm100::prefetch_tmap(&tmW);
    }
    // Under programmatic dependent launch this part overlaps the previous kernel: an L2
    // prefetch of the first weight stages is safe before the dependency is resolved
    // (L2 stays coherent with the previous kernel's writes); the copies into shared
    // memory are issued only after griddepcontrol.wait.
    for (int j = 0; j < a.l2pf && j < nst; ++j)
      sm100::tma_prefetch_l2_2d(&tmW, strip * 32, (b0 + j * kBlocksPerStage) * 8);
  }
  sm100::grid_dependency_wait();        // no-op unless launched as a programmatic dependent
  sm100::grid_launch_dependents();
  __syncwarp();
  if (lane == 0) {
    for (int j = 0; j < kStages && j < nst; ++j) {
      sm100::mbar_arrive_expect_tx(full_bar(warp, j), kStageBytes);
      sm100::tma_load_2d(stage_addr(warp, j), &tmW, full_bar(warp, j), strip * 32,
                         (b0 + j * kBlocksPerStage) * 8);
    }
  }

  // ---- stage activations xs[m][k] and the strip's zeros / scales ---------------------
  // asynchronous 16-byte copies: every thread's copies are in flight at once, so the
  // staging costs one memory round trip (it overlaps the first weight stages)
  {
    const int vecs = Kc / 8;                         // 16-byte vectors per token row
    for (int i = tid; i < MP * vecs; i += kThreads) {
      const int m = i / vecs, v = i - m * vecs;
      const uint32_t dst = sbase + off_xs + (uint32_t)(m * a.xs_stride + v * 8) * 2u;
      if (m < Mc)
        cp_async16(dst, a.x + (int64_t)(m0 + m) * a.ldx + krow0 + v * 8);
      else
        sts128_zero(dst);
    }
    const int g0 = krow0 / a.gs;
    const int ng = Kc > 0 ? (krow0 + Kc - 1) / a.gs - g0 + 1 : 0;
    for (int i = tid; i < ng * 40; i += kThreads) {
      const int gi = i / 40, v = i - gi * 40;      // 8 vectors of zeros, 32 of scales
      if (v < 8) {
        const int wc = strip * 32 + v * 4;
        const uint32_t dst = sbase + off_zs + (uint32_t)(gi * 128 + v * 16);
        if (wc < a.PN) cp_async16(dst, a.qz + (int64_t)(g0 + gi) * a.PN + wc);
        else sts128_zero(dst);
      } else {
        const int n = strip * kStripN + (v - 8) * 8;
        const uint32_t dst = sbase + off_ss + (uint32_t)(gi * kStripN * 2 + (v - 8) * 16);
        if (n < a.N) cp_async16(dst, a.scales + (int64_t)(g0 + gi) * a.N + n);
        else sts128_zero(dst);
      }
    }
    cp_async_wait_all();
  }
  __syncthreads();
  const int grp0 = krow0 / a.gs;

  const int chunk = (g >> 1) | ((g & 1) << 2);       // conflict-free word chunk
  float acc[TOKSETS][8][4];
#pragma unroll
  for (int s2 = 0; s2 < TOKSETS; ++s2)
#pragma unroll
    for (int q = 0; q < 8; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s2][q][i] = 0.f;

  {
    const uint32_t bsel = (g & 1) ? 0x1054u : 0x5410u;   // x into this lane's pair slot
    const uint32_t lane_off_a = (uint32_t)t * 128u + ((uint32_t)(chunk ^ t) << 4);
    const uint32_t lane_off_b = (uint32_t)(t + 4) * 128u + ((uint32_t)(chunk ^ (t + 4)) << 4);
    // shared-memory byte address of x[token][k = 0] for this lane's tokens (k is added
    // per block); explicit ld.shared keeps these loads off the L1TEX path
    uint32_t xrow[TOKSETS];
#pragma unroll
    for (int s2 = 0; s2 < TOKSETS; ++s2)
      xrow[s2] = sbase + off_xs + (uint32_t)(((4 * s2 + (g >> 1)) * a.xs_stride + t - krow0) * 2);
    uint32_t zcst[4][4], scl[4][4];
    float pacc[BIAS ? 8 : 1][4];
    int j = 0;                                          // stage counter of this warp
    bool ok = true;
    for (int kb = b0 * 8; kb < b1 * 8 && ok;) {
      const int grp = kb / a.gs;
      const int kend = min(b1 * 8, (grp + 1) * a.gs);
      const int gl = grp - grp0;
      if constexpr (!BIAS) {
        // fp16 W path: zeros and scales are used per weight
        const uint4 z4 = lds128(sbase + off_zs + (uint32_t)(gl * 128 + chunk * 16));
        const uint32_t zw[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          zero_consts(zw[c], zcst[c]);
          const uint4 s4 = lds128(sbase + off_ss + (uint32_t)(gl * kStripN * 2 + (chunk * 4 + c) * 16));
          scl[c][0] = s4.x; scl[c][1] = s4.y; scl[c][2] = s4.z; scl[c][3] = s4.w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
          for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;
      }
      const int nseg = (kend - kb) / kRowsPerStage;
      for (int i = 0; i < nseg; ++i, ++j) {
        const int s = j % kStages;
        if (!sm100::mbar_wait_bounded(full_bar(warp, s), (j / kStages) & 1, a.status)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        const uint32_t st = stage_addr(warp, s);
        const int krow = kb + i * kRowsPerStage;
#pragma unroll
        for (int h = 0; h < kBlocksPerStage; ++h) {
          const uint4 va = lds128(st + h * 1024 + lane_off_a);
          const uint4 vb = lds128(st + h * 1024 + lane_off_b);
          uint32_t bf0[TOKSETS], bf1[TOKSETS];
#pragma unroll
          for (int s2 = 0; s2 < TOKSETS; ++s2) {
            const uint32_t xa = xrow[s2] + (uint32_t)(krow + h * 8) * 2u;
            bf0[s2] = prmt(lds_u16(xa), 0u, bsel);
            bf1[s2] = prmt(lds_u16(xa + 8u), 0u, bsel);
          }
          const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
          const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t da[4], db[4];
            if constexpr (BIAS) {
              unpack_biased(wa[c], da);
              unpack_biased(wb[c], db);
            } else {
              dequant_word(wa[c], zcst[c], scl[c], da);
              dequant_word(wb[c], zcst[c], scl[c], db);
            }
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int q = 2 * c + jj;
              if constexpr (BIAS) {
                mma_16816(pacc[q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf0[0],
                          bf1[0]);
              } else {
#pragma unroll
                for (int s2 = 0; s2 < TOKSETS; ++s2)
                  mma_16816(acc[s2][q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1],
                            bf0[s2], bf1[s2]);
              }
            }
          }
        }
        // refill this stage with stage j + kStages: every lane's loads from it were
        // consumed by the MMAs above
        __syncwarp();
        if (lane == 0 && j + kStages < nst) {
          sm100::mbar_arrive_expect_tx(full_bar(warp, s), kStageBytes);
          sm100::tma_load_2d(st, &tmW, full_bar(warp, s), strip * 32,
                             (b0 + (j + kStages) * kBlocksPerStage) * 8);
        }
      }
      if constexpr (BIAS) {
        // close the group segment [kb, kend): remove the zero term, apply the scale
        float part = 0.f;
        const int u0 = (kb - krow0) >> 3, u1 = (kend - krow0) >> 3;
        const uint32_t xt = sbase + off_xs + (uint32_t)(t * a.xs_stride) * 2u;
        for (int u = u0 + g; u < u1; u += 8) {
          const uint4 v = lds128(xt + (uint32_t)u * 16u);
          const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(u32_as_h2(hv[k]));
            part += f.x + f.y;
          }
        }
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        part += __shfl_xor_sync(0xffffffffu, part, 8);
        part += __shfl_xor_sync(0xffffffffu, part, 16);   // sum(x[token t]) over the segment
        const uint4 z4 = lds128(sbase + off_zs + (uint32_t)(gl * 128 + chunk * 16));
        const uint32_t zw[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 s4 = lds128(sbase + off_ss + (uint32_t)(gl * kStripN * 2 + (chunk * 4 + c) * 16));
          const uint32_t sv[4] = {s4.x, s4.y, s4.z, s4.w};
          const uint32_t z8 = zw[c] >> 8;
          const uint32_t zb[4] = {lop3_and_or(zw[c], kLoMask, kMagic),   // 1024 + z
                                  lop3_and_or(zw[c], kHiMask, kMagic),   // 1024 + 16 z
                                  lop3_and_or(z8, kLoMask, kMagic),
                                  lop3_and_or(z8, kHiMask, kMagic)};
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int q = 2 * c + jj;
            const float2 zl = __half22float2(u32_as_h2(zb[2 * jj]));
            const float2 zh = __half22float2(u32_as_h2(zb[2 * jj + 1]));
            const float2 sl = __half22float2(u32_as_h2(sv[2 * jj]));
            const float2 sh = __half22float2(u32_as_h2(sv[2 * jj + 1]));
            acc[0][q][0] = fmaf(sl.x, fmaf(-zl.x, part, pacc[q][0]), acc[0][q][0]);
            acc[0][q][1] = fmaf(sl.y, fmaf(-zl.y, part, pacc[q][1]), acc[0][q][1]);
            acc[0][q][2] = fmaf(sh.x * 0.0625f, fmaf(-zh.x, part, pacc[q][2]), acc[0][q][2]);
            acc[0][q][3] = fmaf(sh.y * 0.0625f, fmaf(-zh.y, part, pacc[q][3]), acc[0][q][3]);
          }
        }
      }
      kb = kend;
    }
    if (!ok && lane == 0) {
      // a stage never arrived: wait (bounded) for this warp's copies still in flight
      for (int jj = j; jj < nst && jj < j + kStages; ++jj)
        sm100::mbar_wait_bounded(full_bar(warp, jj % kStages), (jj / kStages) & 1, nullptr,
                                 50000000ull);
    }
    __syncwarp();
  }

  // ---- CTA reduction: each warp parks its partial in its own (now idle) ring, one
  // barrier, then the 8 partials are summed in warp order -------------------------------
  {
    float* mine = reinterpret_cast<float*>(sgen + (uint32_t)warp * kStages * kStageBytes);
#pragma unroll
    for (int s2 = 0; s2 < TOKSETS; ++s2) {
      const int m = 4 * s2 + t;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(mine + m * DecGeo<TOKSETS>::kPartStride + 32 * chunk + 4 * q) =
            make_float4(acc[s2][q][0], acc[s2][q][1], acc[s2][q][2], acc[s2][q][3]);
    }
  }
  __syncthreads();
  const int nbase = strip * kStripN;
  for (int idx = tid; idx < MP * kStripN; idx += kThreads) {
    const int m = idx / kStripN, nl = idx - m * kStripN;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w)
      v += reinterpret_cast<const float*>(sgen + (uint32_t)w * kStages * kStageBytes)
               [m * DecGeo<TOKSETS>::kPartStride + nl];
    if (a.cs == 1) {
      const int n = nbase + nl;
      if (m < Mc && n < a.N) a.out[(int64_t)(m0 + m) * a.ldo + n] = __float2half_rn(v);
    } else {
      red[m * kRedStride + nl] = v;
    }
  }
  if (a.cs == 1) return;                               // grid-uniform: no cluster to serve

  // ---- cluster reduction over distributed shared memory ----------------------------
  cluster_sync_all();                                  // every CTA's red is complete
  const int cw = kStripN / a.cs;                       // columns reduced by this CTA
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

struct TmaPlan {
  int cs, bps, xs_stride, ngrp, toksets;
  size_t smem;
};

template <int TOKSETS>
size_t smem_bytes(int xs_stride, int ngrp) {
  const int MP = 4 * TOKSETS;
  constexpr int S = DecGeo<TOKSETS>::kStages;
  return 1024 + DecGeo<TOKSETS>::kRingBytes + (size_t)MP * kRedStride * 4 +
         kConsumers * S * 8 + 16 + (size_t)MP * xs_stride * 2 + (size_t)ngrp * (128 + kStripN * 2);
}

// Cluster size: grow the split-K factor while the grid stays within one CTA per SM and
// every consumer warp keeps at least two stages; then grow it further (up to max_cs)
// if the CTA's staged activations do not fit in shared memory.
bool plan_tma(int64_t M, int64_t N, int64_t K, int64_t gs, int num_sms, int max_cs, TmaPlan* p) {
  if (N % 32 || gs % kRowsPerStage || K % gs) return false;
  const int64_t strips = (N + kStripN - 1) / kStripN;
  // M <= 4: one 4-token set; otherwise chunks of 8 tokens (two sets) per CTA row of the
  // grid -- 16 tokens per CTA would need more registers than 9 warps per SM allow
  p->toksets = M <= 4 ? 1 : 2;
  const int64_t zchunks = (M + 4 * p->toksets - 1) / (4 * p->toksets);
  const int64_t KB = K / 8;
  int cs = 1;
  while (cs < max_cs && strips * zchunks * cs * 2 <= (int64_t)num_sms &&
         KB / (cs * 2) >= (int64_t)kConsumers * kBlocksPerStage * 2)
    cs *= 2;
  for (;; cs *= 2) {
    int bps = (int)((KB + cs - 1) / cs);
    bps = (bps + kBlocksPerStage - 1) / kBlocksPerStage * kBlocksPerStage;
    const int xs_stride = bps * 8 + 8;                // +16 B staggers token rows
    const int ngrp = (int)((bps * 8 + gs - 1) / gs) + 1;
    size_t smem = p->toksets == 1 ? smem_bytes<1>(xs_stride, ngrp) : smem_bytes<2>(xs_stride, ngrp);
    if (smem <= kGemvTmaMaxSmem) {
      p->cs = cs; p->bps = bps; p->xs_stride = xs_stride; p->ngrp = ngrp; p->smem = smem;
      return true;
    }
    if (cs >= max_cs) return false;
  }
}

// Programmatic dependent launch is off unless AWQ_PDL=1 (read once per process): on the
// mixed decode stack it measured slower than plain stream order.
bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AWQ_PDL");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

template <int TOKSETS>
cudaError_t launch_t(const CUtensorMap& tm, const TmaGemvArgs& a, int strips, int zchunks,
                     size_t smem, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(gemv_tma_kernel<TOKSETS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvTmaMaxSmem);
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
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.cs;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  // programmatic dependent launch: the kernel waits (griddepcontrol.wait) before it
  // touches anything the previous grid may write
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<TOKSETS>, tm, a);
}

}  // namespace

bool gemv_tma_supported(const int32_t* qweight, int64_t N, int64_t ldx, const void* x) {
  return (N % 32 == 0) && ((reinterpret_cast<uintptr_t>(qweight) & 15) == 0) &&
         ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 8 == 0) && encode_fn() != nullptr;
}

int gemv_tma_cluster_size(int64_t M, int64_t N, int64_t K, int num_sms, int max_cs) {
  TmaPlan p;
  if (!plan_tma(M, N, K, 128, num_sms, max_cs, &p)) return 0;
  return p.cs;
}

size_t gemv_tma_smem_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                           int max_cs) {
  TmaPlan p;
  if (!plan_tma(M, N, K, group_size, num_sms, max_cs, &p)) return (size_t)-1;
  return p.smem;
}

cudaError_t launch_gemv_tma(const void* x, int64_t ldx, const int32_t* qweight,
                            const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                            int M, int N, int K, int group_size, int num_sms, int max_cs,
                            int* dev_status, cudaStream_t stream) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  TmaPlan p;
  if (!plan_tma(M, N, K, group_size, num_sms, max_cs, &p)) return cudaErrorInvalidValue;
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)(N / 8), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)N / 2};
  cuuint32_t box[2] = {32, (cuuint32_t)kRowsPerStage};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const int strips = (N + kStripN - 1) / kStripN;
  TmaGemvArgs a;
  a.ldx = ldx;
  a.qz = qzeros;
  a.scales = static_cast<const __half*>(scales);
  a.ldo = ldo;
  a.N = N; a.K = K; a.gs = group_size; a.PN = N / 8; a.KB = K / 8;
  a.cs = p.cs;
  a.bps = p.bps;
  a.xs_stride = p.xs_stride;
  a.ngrp_cta = p.ngrp;
  a.l2pf = pdl_enabled() ? 4 : 0;
  a.status = dev_status;
  const int64_t chunk = 4 * p.toksets;                 // tokens per CTA row of the grid
  const int64_t max_rows = (int64_t)65535 * chunk;
  for (int64_t m0 = 0; m0 < M; m0 += max_rows) {
    const int64_t rows = (M - m0 < max_rows) ? (M - m0) : max_rows;
    a.x = static_cast<const __half*>(x) + m0 * ldx;
    a.out = static_cast<__half*>(out) + m0 * ldo;
    a.M = (int)rows;
    const int z = (int)((rows + chunk - 1) / chunk);
    cudaError_t e = p.toksets == 1 ? launch_t<1>(tm, a, strips, z, p.smem, stream)
                                   : launch_t<2>(tm, a, strips, z, p.smem, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace awq
