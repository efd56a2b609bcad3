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

#include <cstdlib>
#include <mutex>

#include "awq_common.cuh"
#include "awq_internal.h"
#include "awq_sm100.cuh"

namespace awq {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;                 // per-warp ring depth
constexpr int kRowsPerStage = 16;          // two 8-row blocks per TMA copy
constexpr int kStripN = 256;
constexpr uint32_t kStageBytes = kRowsPerStage * 128;                // 2 KB
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
  int bps;         // 8-row blocks per CTA (even)
  int xs_stride;   // halves per token row of xs
  int ngrp_cta;    // quantization groups a CTA's K range can touch (zs / ss rows)
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

// Biased unpack: 4 half2 holding (1024 + w) for nibbles at bits 0..3 / 16..19 and
// (1024 + 16 w) for bits 4..7 / 20..23, of the word and of word >> 8 -- exact values,
// element pairs (0,1), (2,3), (4,5), (6,7).  No zero subtraction per weight.
// `magic` (0x64006400) arrives in a register whose value the compiler cannot see, so
// each lop3 keeps one immediate (the mask) and one register operand and stays a single
// instruction.
__device__ __forceinline__ void unpack_biased(uint32_t w, uint32_t magic, uint32_t d[4]) {
#if AWQ_DEC_OPAQUE == 0
  const uint32_t w8 = w >> 8;
  d[0] = lop3_and_or(w, kLoMask, kMagic);
  d[1] = lop3_and_or(w, kHiMask, kMagic);
  d[2] = lop3_and_or(w8, kLoMask, kMagic);
  d[3] = lop3_and_or(w8, kHiMask, kMagic);
#elif AWQ_DEC_OPAQUE == 1
  const uint32_t w8 = w >> 8;
  d[0] = lop3_and_or(w, kLoMask, magic);
  d[1] = lop3_and_or(w, kHiMask, magic);
  d[2] = lop3_and_or(w8, kLoMask, magic);
  d[3] = lop3_and_or(w8, kHiMask, magic);
#else
  const uint32_t w8 = w >> 8;
  const uint32_t lo = magic >> 16, hi = lo << 4;   // opaque masks too: 0x6400 -> not used
  d[0] = lop3_and_or(w, kLoMask, magic);
  d[1] = lop3_and_or(w, kHiMask, magic);
  d[2] = lop3_and_or(w8, kLoMask, magic);
  d[3] = lop3_and_or(w8, kHiMask, magic);
  (void)lo; (void)hi;
#endif
}
__device__ __forceinline__ uint32_t opaque_u32(uint32_t v) {
  uint32_t r;
  asm volatile("mov.b32 %0, %1;" : "=r"(r) : "r"(v));
  return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Tuning knobs (compile time): CTAs per SM the M<=4 variant is built for (register
// budget 65536 / (256 * AWQ_DEC_MINB)), and how many stages each warp prefetches into L2
// before the grid dependency wait.
#ifndef AWQ_DEC_MINB
#define AWQ_DEC_MINB 2
#endif
#ifndef AWQ_DEC_L2PF
#define AWQ_DEC_L2PF 0
#endif
#ifndef AWQ_DEC_OPAQUE
#define AWQ_DEC_OPAQUE 1
#endif

template <int TOKSETS>
__global__ void __launch_bounds__(kThreads, TOKSETS == 1 ? AWQ_DEC_MINB : 1)
gemv_tma_kernel(const __grid_constant__ CUtensorMap tmW, const TmaGemvArgs a) {
  constexpr int MP = 4 * TOKSETS;
  // BIAS (one 4-token set): the MMAs accumulate x * (1024 + w) / x * (1024 + 16 w)
  // over one quantization group; at the group's end the exact zero term
  // (1024 + z) * sum(x) (resp. (1024 + 16 z) * sum(x)) is removed and the fp32 scale
  // (resp. scale / 16) applied.  For more tokens W is rounded to fp16 first exactly
  // as the reference does, and the MMA accumulates x * W directly.
  constexpr bool BIAS = (TOKSETS == 1);
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;
  unsigned char* sgen = smem_raw + (sbase - base_raw);
  // layout: ring | red (MP x 264 fp32) | bars (kWarps x kStages) | xs | zs | ss
  const uint32_t off_red = kRingBytes;
  const uint32_t off_bar = off_red + MP * kRedStride * 4;
  const uint32_t off_xs = off_bar + kWarps * kStages * 8;
  const uint32_t off_zs = off_xs + (uint32_t)MP * a.xs_stride * 2;
  const uint32_t off_ss = off_zs + (uint32_t)a.ngrp_cta * 128;
  float* red = reinterpret_cast<float*>(sgen + off_red);
  __half* xs = reinterpret_cast<__half*>(sgen + off_xs);
  uint32_t* zs = reinterpret_cast<uint32_t*>(sgen + off_zs);    // [group][32 words]
  __half* ss = reinterpret_cast<__half*>(sgen + off_ss);        // [group][256]

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
  int per = (nb + kWarps - 1) / kWarps;
  per += per & 1;                                    // whole stages per warp
  const int b0 = cb0 + min(nb, warp * per);
  const int b1 = cb0 + min(nb, (warp + 1) * per);
  const int nblk = b1 - b0;
  const int nst = (nblk + 1) >> 1;                   // stages this warp consumes
  const int krow0 = cb0 * 8;
  const int Kc = nb * 8;

  const uint32_t ring = sbase + (uint32_t)warp * kStages * kStageBytes;
  const uint32_t bars = sbase + off_bar + (uint32_t)warp * kStages * 8;

  // ---- barriers, L2 prefetch of the first tiles, then wait for the previous grid -----
  // Under programmatic dependent launch this prologue overlaps the tail of the
  // preceding kernel; nothing below griddepcontrol.wait reads memory it may write.
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) sm100::mbar_init(bars + 8 * s, 1);
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmW);
    for (int j = 0; j < AWQ_DEC_L2PF && j < nst; ++j)
      sm100::tma_prefetch_l2_2d(&tmW, strip * 32, (b0 + 2 * j) * 8);
  }
  sm100::grid_dependency_wait();
  sm100::grid_launch_dependents();
  __syncwarp();
  if (lane == 0) {
    for (int j = 0; j < kStages && j < nst; ++j) {
      sm100::mbar_arrive_expect_tx(bars + 8 * j, kStageBytes);
      sm100::tma_load_2d(ring + j * kStageBytes, &tmW, bars + 8 * j, strip * 32, (b0 + 2 * j) * 8);
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
    // zeros (32 words) and scales (256 fp16) of the strip for the CTA's groups
    const int g0 = krow0 / a.gs;
    const int ng = Kc > 0 ? (krow0 + Kc - 1) / a.gs - g0 + 1 : 0;
    for (int i = tid; i < ng * 40; i += kThreads) {
      const int gi = i / 40, v = i - gi * 40;     // 8 vectors of zeros, 32 of scales
      uint4 val = make_uint4(0, 0, 0, 0);
      if (v < 8) {
        const int wc = strip * 32 + v * 4;
        if (wc < a.PN) val = __ldg(reinterpret_cast<const uint4*>(a.qz + (int64_t)(g0 + gi) * a.PN + wc));
        reinterpret_cast<uint4*>(zs + gi * 32)[v] = val;
      } else {
        const int n = strip * kStripN + (v - 8) * 8;
        if (n < a.N) val = __ldg(reinterpret_cast<const uint4*>(a.scales + (int64_t)(g0 + gi) * a.N + n));
        reinterpret_cast<uint4*>(ss + gi * kStripN)[v - 8] = val;
      }
    }
  }
  __syncthreads();
  const int grp0 = krow0 / a.gs;                      // first group staged in zs / ss

  const uint32_t magic = opaque_u32(kMagic);
  const int chunk = (g >> 1) | ((g & 1) << 2);       // conflict-free word chunk
  // B column g = (token g/2, pair slot g%2): x goes to the low half for slot 0 and
  // to the high half for slot 1 (prmt selector; bytes 4..7 come from the zero word)
  const uint32_t bsel = (g & 1) ? 0x1054u : 0x5410u;
  const int wc0 = strip * 32 + chunk * 4;            // first packed word of this lane
  float acc[TOKSETS][8][4];
#pragma unroll
  for (int s = 0; s < TOKSETS; ++s)
#pragma unroll
    for (int q = 0; q < 8; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][q][i] = 0.f;
  float pacc[BIAS ? 8 : 1][4];
#pragma unroll
  for (int q = 0; q < (BIAS ? 8 : 1); ++q)
#pragma unroll
    for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;

  uint32_t zcst[4][4], scl[4][4];
  int grp_end = -1, seg_k0 = 0;
  // close the segment [seg_k0, kend) of the current group (BIAS path)
  auto flush = [&](int kend) {
    if constexpr (BIAS) {
      // zeros and scales of the group being closed, from the CTA's shared-memory copy
      const int gl = seg_k0 / a.gs - grp0;
      const uint4 z4 = reinterpret_cast<const uint4*>(zs + gl * 32)[chunk];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 s4 = reinterpret_cast<const uint4*>(ss + gl * kStripN)[chunk * 4 + c];
        scl[c][0] = s4.x; scl[c][1] = s4.y; scl[c][2] = s4.z; scl[c][3] = s4.w;
      }
      const uint32_t zw[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t z8 = zw[c] >> 8;
        zcst[c][0] = lop3_and_or(zw[c], kLoMask, kMagic);
        zcst[c][1] = lop3_and_or(zw[c], kHiMask, kMagic);
        zcst[c][2] = lop3_and_or(z8, kLoMask, kMagic);
        zcst[c][3] = lop3_and_or(z8, kHiMask, kMagic);
      }
      float part = 0.f;
      const int u0 = (seg_k0 - krow0) >> 3, u1 = (kend - krow0) >> 3;
      for (int u = u0 + g; u < u1; u += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xs + t * a.xs_stride + u * 8);
        const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(u32_as_h2(hv[j]));
          part += f.x + f.y;
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      part += __shfl_xor_sync(0xffffffffu, part, 8);
      part += __shfl_xor_sync(0xffffffffu, part, 16);    // sum(x[token t]) over the segment
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = q >> 1, jj = q & 1;
        const float2 zl = __half22float2(u32_as_h2(zcst[c][2 * jj]));       // 1024 + z
        const float2 zh = __half22float2(u32_as_h2(zcst[c][2 * jj + 1]));   // 1024 + 16 z
        const float2 sl = __half22float2(u32_as_h2(scl[c][2 * jj]));
        const float2 sh = __half22float2(u32_as_h2(scl[c][2 * jj + 1]));
        acc[0][q][0] = fmaf(sl.x, fmaf(-zl.x, part, pacc[q][0]), acc[0][q][0]);
        acc[0][q][1] = fmaf(sl.y, fmaf(-zl.y, part, pacc[q][1]), acc[0][q][1]);
        acc[0][q][2] = fmaf(sh.x * 0.0625f, fmaf(-zh.x, part, pacc[q][2]), acc[0][q][2]);
        acc[0][q][3] = fmaf(sh.y * 0.0625f, fmaf(-zh.y, part, pacc[q][3]), acc[0][q][3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) pacc[q][i] = 0.f;
      }
    }
    seg_k0 = kend;
  };

  int j_fail = nst;                     // first stage that never arrived
  for (int j = 0; j < nst; ++j) {
    const int s = j % kStages;
    if (!sm100::mbar_wait_bounded(bars + 8 * s, (j / kStages) & 1, a.status)) {
      j_fail = j;
      break;
    }
    const uint32_t st = ring + s * kStageBytes;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int bb = b0 + 2 * j + h;
      if (bb < b1) {
        // rows t and t+4 of block h: atom h, swizzled 16-byte chunk
        const uint4 va = lds128(st + h * 1024 + t * 128 + ((uint32_t)(chunk ^ t) << 4));
        const uint4 vb = lds128(st + h * 1024 + (t + 4) * 128 + ((uint32_t)(chunk ^ (t + 4)) << 4));
        const int k0 = bb * 8;
        if (k0 >= grp_end) {
          if (grp_end >= 0) flush(k0);
          const int grp = k0 / a.gs;
          grp_end = (grp + 1) * a.gs;
          seg_k0 = k0;
          if constexpr (!BIAS) {
            // fp16 W path: zeros and scales are used per weight
            const int gl = grp - grp0;
            const uint4 z4 = reinterpret_cast<const uint4*>(zs + gl * 32)[chunk];
            const uint32_t zw[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              zero_consts(zw[c], zcst[c]);
              const uint4 s4 = reinterpret_cast<const uint4*>(ss + gl * kStripN)[chunk * 4 + c];
              scl[c][0] = s4.x; scl[c][1] = s4.y; scl[c][2] = s4.z; scl[c][3] = s4.w;
            }
          }
        }
        uint32_t bf0[TOKSETS], bf1[TOKSETS];
        const int kl = k0 - krow0;
#pragma unroll
        for (int s2 = 0; s2 < TOKSETS; ++s2) {
          const __half* xp = xs + (4 * s2 + (g >> 1)) * a.xs_stride + kl + t;
          const uint32_t xa = __half_as_ushort(xp[0]);
          const uint32_t xb = __half_as_ushort(xp[4]);
          bf0[s2] = prmt(xa, 0u, bsel);          // x in the slot of this lane's column
          bf1[s2] = prmt(xb, 0u, bsel);
        }
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
        const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t da[4], db[4];
          if constexpr (BIAS) {
            unpack_biased(wa[c], magic, da);
            unpack_biased(wb[c], magic, db);
          } else {
            dequant_word(wa[c], zcst[c], scl[c], da);
            dequant_word(wb[c], zcst[c], scl[c], db);
          }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int q = 2 * c + jj;
            if constexpr (BIAS) {
              mma_16816(pacc[q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf0[0], bf1[0]);
            } else {
#pragma unroll
              for (int s2 = 0; s2 < TOKSETS; ++s2)
                mma_16816(acc[s2][q], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1],
                          bf0[s2], bf1[s2]);
            }
          }
        }
      }
    }
    // refill this stage with stage j + kStages: every lane's reads of it have completed
    // (their values were consumed above), so the copy may overwrite it
    __syncwarp();
    if (lane == 0 && j + kStages < nst) {
      sm100::mbar_arrive_expect_tx(bars + 8 * s, kStageBytes);
      sm100::tma_load_2d(st, &tmW, bars + 8 * s, strip * 32, (b0 + 2 * (j + kStages)) * 8);
    }
  }
  if (grp_end >= 0) flush(min(b1 * 8, grp_end));
  if (j_fail < nst && lane == 0) {
    // a stage never arrived: wait (bounded) for the copies this warp still has in
    // flight -- stages [j_fail, j_fail + kStages) -- before the CTA may exit
    for (int j = j_fail; j < nst && j < j_fail + kStages; ++j)
      sm100::mbar_wait_bounded(bars + 8 * (j % kStages), (j / kStages) & 1, nullptr, 50000000ull);
  }
  __syncwarp();

  // ---- CTA reduction: warps add into red[m][n] in fixed order ----------------------
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int s2 = 0; s2 < TOKSETS; ++s2) {
        const int m = 4 * s2 + t;
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
size_t smem_bytes(int xs_stride, int ngrp) {
  const int MP = 4 * TOKSETS;
  return 1024 + kRingBytes + (size_t)MP * kRedStride * 4 + kWarps * kStages * 8 +
         (size_t)MP * xs_stride * 2 + (size_t)ngrp * (128 + kStripN * 2);
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
  cuuint32_t box[2] = {32, (cuuint32_t)kRowsPerStage};
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
  a.bps += a.bps & 1;                                  // whole 16-row stages
  a.xs_stride = a.bps * 8 + 8;                        // +16 B staggers token rows
  a.ngrp_cta = (a.bps * 8 + group_size - 1) / group_size + 1;
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
      case 1: e = launch_t<1>(tm, a, strips, z, smem_bytes<1>(a.xs_stride, a.ngrp_cta), stream); break;
      case 2: e = launch_t<2>(tm, a, strips, z, smem_bytes<2>(a.xs_stride, a.ngrp_cta), stream); break;
      default: e = launch_t<4>(tm, a, strips, z, smem_bytes<4>(a.xs_stride, a.ngrp_cta), stream); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t gemv_tma_smem_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                           int max_cs) {
  const int cs = gemv_tma_cluster_size(M < 16 ? M : 16, N, K, num_sms, max_cs);
  int bps = (int)((K / 8 + cs - 1) / cs);
  bps += bps & 1;
  const int mc = M < 16 ? (int)M : 16;
  const int xs_stride = bps * 8 + 8;
  const int ngrp = (int)((bps * 8 + group_size - 1) / group_size) + 1;
  return mc <= 4 ? smem_bytes<1>(xs_stride, ngrp)
                 : (mc <= 8 ? smem_bytes<2>(xs_stride, ngrp) : smem_bytes<4>(xs_stride, ngrp));
}

}  // namespace awq
