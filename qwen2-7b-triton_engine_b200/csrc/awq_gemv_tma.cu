// awq_gemv_tma.cu -- decode AWQ W4A16 product (M <= 16 per launch), TMA-streamed, one
// CTA per SM, deterministic split-K.  The fast path of the decode branch; awq_gemv.cu
// keeps the generic kernel for shapes TMA cannot describe (N % 32 != 0,
// group_size % 32 != 0, unaligned pointers).
//
// Replaces the M <= 4 dequant + torch.matmul branch of awq_gemm_forward
// (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:251-266) and small-M calls
// of _awq_gemm_kernel (kernels/awq_gemm.py:152-228).
//
// Work split
//   An output tile is one 256-column strip of one chunk of 4 (M <= 4) or 8 tokens.  The
//   grid has one CTA per SM whenever the tiles allow it: each tile gets `base` or
//   `base + 1` CTAs, and each of those streams a contiguous, stage-aligned K range of
//   the tile (the ranges of one tile differ by at most one 32-row stage), so every SM
//   streams about the same number of bytes.
// Roles (one CTA = 8 warps)
//   every warp owns a contiguous, stage-aligned part of the CTA's K range and a ring of
//   two 8 KB shared-memory stages it refills itself: one 2-D TMA load of 64 K-rows x 32
//   packed words (128-byte swizzle) per stage, completing on the stage's mbarrier.  It
//   walks its range one quantization group at a time; the inner loop over the group's
//   stages is branch-free apart from the barrier wait and the refill: 8 x (2 shared
//   loads + biased unpack + 8 mma.sync) per stage.  The group's zero/scale correction
//   runs once per group, outside that loop.
//   lane (g = lane/4, t = lane%4) reads rows t and t+4 of each 8-row block as 16 bytes
//   from word chunk c(g) = (g >> 1) | ((g & 1) << 2); with the swizzle (chunk ^ row)
//   the 8 lanes of each shared-memory phase hit 8 distinct 16-byte bank groups.
// Prologue
//   before griddepcontrol.wait (overlapping the previous kernel under programmatic
//   launch): barrier set-up and an L2 prefetch of every warp's first weight stages.
//   After it: all threads cp.async-copy the activations into shared memory, every warp
//   issues its first weight stages and cp.async-copies the zero / scale rows of its own
//   groups; the loop starts on the activations alone.
// Math: dequantized pairs feed mma.sync.m16n8k16 (fp16 x fp16 -> fp32) with the
//   activations spread over the (token, pair-slot) B columns.  For M <= 4 the MMA takes
//   the exact biased values 1024 + w / 1024 + 16 w; each group segment's fp32 accumulator
//   starts at -(1024 + z) * sum(x) (resp. -(1024 + 16 z) * sum(x)), computed while the
//   segment's stages are in flight, and the fp32 scale (scale / 16) is applied when the
//   segment closes; for M > 4 W is rounded to fp16 first exactly as the reference does.
// Split-K: each CTA sums its 8 warps' partials in shared memory (fixed order).  A tile
//   with one CTA writes fp16 directly.  Otherwise each CTA writes an fp32 partial into
//   its own workspace slot, and the last CTA of the tile to take a ticket (an acq_rel
//   atomic counter, which that CTA resets) sums the tile's slots in slot order --
//   deterministic -- and writes fp16.
// Every mbarrier wait is bounded (status word + early exit, after a bounded drain of
// the copies still in flight).
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
constexpr int kRowsPerStage = 64;                 // eight 8-row blocks per TMA copy
constexpr int kBlocksPerStage = kRowsPerStage / 8;
constexpr int kStripN = 256;
constexpr uint32_t kStageBytes = kRowsPerStage * 128;                // 8 KB
// per-warp ring depth: 8 warps x 2 x 8 KB = 128 KB of weight copies in flight per SM.
// 8 KB copies: the TMA unit's cost per copy made 4 KB copies measurably slower.  One CTA
// per SM: with two, the block scheduler was seen packing two CTAs of one call onto one
// SM while other SMs idled.
constexpr int kStages = 2;
constexpr uint32_t kRingBytes = kConsumers * kStages * kStageBytes;
constexpr int kMaxSplits = 32;                    // CTAs per output tile, at most
constexpr int kMinStagesPerCta = 1;               // K rows per CTA, at least one stage
// Weight stages per warp that are prefetched into L2 before the dependency wait.
constexpr int kL2PrefetchStages = 2;

template <int TOKSETS>
struct DecGeo {
  // row stride (floats) of a warp's partial sums parked in its own ring after the loop;
  // MP rows of it must fit the warp's kStages * 4 KB
  static constexpr int kPartStride = TOKSETS == 1 ? 264 : kStripN;
  static_assert(4 * TOKSETS * kPartStride * 4 <= kStages * (int)kStageBytes, "partials fit the ring");
};

struct TmaGemvArgs {
  const __half* x;
  int64_t ldx;
  const int32_t* qw;
  const int32_t* qz;
  const __half* scales;
  __half* out;
  int64_t ldo;
  float* part;     // split-K partial slots [cta][MP][256] fp32 (null when no tile is split)
  int* cnt;        // arrival counter per tile, zero between calls (null when no split)
  int M, N, K, gs, PN, KB;
  int strips;      // 256-column strips; tile = strip + strips * token chunk
  int base, extra; // CTAs per tile: tiles [0, extra) get base + 1, the others base
  int xs_stride;   // halves per token row of xs
  int xr;          // token rows reserved in xs
  int ngrp_cta;    // zs / ss rows reserved (quantization groups a CTA's K range touches)
  int l2pf;        // weight stages each warp prefetches into L2 before the dependency wait
  int* status;
  ArArgs ar;       // fused all-reduce across tensor-parallel ranks (ar.world == 1: none)
  const __half* bias;   // fp16 [N] added to every output row in fp32, or null
  // SiLU-mul epilogue (pair_strips > 0): columns [0, N/2) are gate, [N/2, N) up, and
  // out[m, n] = silu(gate[m, n]) * up[m, n] for n < N/2.  Strip s < pair_strips pairs
  // with strip s + pair_strips; each tile parks its final fp32 values in pair_vals and
  // the second tile of a pair to finish (ticket on pair_cnt) writes the product.
  int pair_strips;
  float* pair_vals;     // [tiles][MP][256] fp32
  int* pair_cnt;        // [token chunks x pair_strips], zero between calls
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

// 16-byte asynchronous global -> shared copy (no register round trip), awaited with
// cp_async_wait_all by the issuing thread.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// One arrival on mbarrier `bar` once all of this thread's earlier cp.async copies have
// landed (the arrival is not counted in advance: the barrier's count includes it).
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared.b64 [%0];" ::"r"(bar) : "memory");
}

// Fused all-reduce: value and flag packed in one aligned 64-bit word (flag in the high
// half), written with one store -- single-copy atomic, so it arrives whole at the
// receiver, local or a peer over NVLink -- and polled with one volatile 64-bit load.
__device__ __forceinline__ void st_pair(unsigned long long* p, float v, uint32_t flag) {
  const unsigned long long w = ((unsigned long long)flag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 ld_pair(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));   // {value bits, flag}
}

// Atomic add at gpu scope with acquire-release ordering; returns the old value.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
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
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;
  unsigned char* sgen = smem_raw + (sbase - base_raw);
  // layout: ring | stage bars | staging bar (x) | flags | xs | zs | ss
  const uint32_t off_full = kRingBytes;
  const uint32_t off_sbar = off_full + kConsumers * kStages * 8;
  const uint32_t off_misc = off_sbar + 16;
  const uint32_t off_xs = off_misc + 16;
  const uint32_t off_zs = off_xs + (uint32_t)a.xr * a.xs_stride * 2;
  const uint32_t off_ss = off_zs + (uint32_t)a.ngrp_cta * 128;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + off_misc);
  volatile int* last_flag = reinterpret_cast<volatile int*>(sgen + off_misc + 4);
  const uint32_t xbar = sbase + off_sbar;          // activations staged

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;

  // ---- this CTA's tile and K range -----------------------------------------------------
  const int cta = blockIdx.x;
  const int big = a.extra * (a.base + 1);
  int tile, split, nsplit, first;
  if (cta < big) {
    tile = cta / (a.base + 1);
    split = cta - tile * (a.base + 1);
    nsplit = a.base + 1;
    first = tile * (a.base + 1);
  } else {
    const int q = (cta - big) / a.base;
    tile = a.extra + q;
    split = cta - big - q * a.base;
    nsplit = a.base;
    first = big + q * a.base;
  }
  const int strip = tile % a.strips;
  const int m0 = (tile / a.strips) * MP;            // token chunk of this CTA
  const int Mc = min(MP, a.M - m0);
  const int nstage_tile = a.KB / kBlocksPerStage;
  const int st0 = (int)((int64_t)split * nstage_tile / nsplit);
  const int st1 = (int)((int64_t)(split + 1) * nstage_tile / nsplit);
  const int cb0 = st0 * kBlocksPerStage;
  const int nb = (st1 - st0) * kBlocksPerStage;
  const int krow0 = cb0 * 8;
  const int Kc = nb * 8;
  const int g0 = krow0 / a.gs;
  const int ng = Kc > 0 ? (krow0 + Kc - 1) / a.gs - g0 + 1 : 0;
  auto full_bar = [&](int w, int s) { return sbase + off_full + (uint32_t)(w * kStages + s) * 8u; };
  auto stage_addr = [&](int w, int s) {
    return sbase + (uint32_t)(w * kStages + s) * kStageBytes;
  };

  int b0, b1;
  warp_range(cb0, nb, warp, b0, b1);
  const int nst = (b1 - b0) / kBlocksPerStage;
  if (lane == 0) {
    for (int s2 = 0; s2 < kStages; ++s2) sm100::mbar_init(full_bar(warp, s2), 1);
    if (warp == 0) {
      sm100::mbar_init(xbar, kThreads);             // one arrival per thread's x copies
      *abort_flag = 0;
      sm100::prefetch_tmap(&tmW);
    }
    sm100::fence_mbar_init();
  }
  __syncthreads();                                   // barriers initialised for every thread
  // ---- before the dependency wait: warm L2 with this warp's first weight stages, one
  // 128-byte row segment per lane and prefetch (plain prefetches: they do not occupy the
  // TMA unit).  The weights are read-only inputs, and a prefetch only fills L2 -- the
  // coherence point -- so it never hands the kernel a stale value; everything that lands
  // in registers or shared memory is read after griddepcontrol.wait.
  for (int j = 0; j < a.l2pf && j < nst; ++j)
#pragma unroll
    for (int r = lane; r < kRowsPerStage; r += 32)
      sm100::prefetch_l2(a.qw + (int64_t)((b0 + j * kBlocksPerStage) * 8 + r) * a.PN + strip * 32);
  sm100::grid_dependency_wait();        // no-op unless launched as a programmatic dependent
  sm100::grid_launch_dependents();

  // ---- staging.  Activations xs[m][k] (Mc rows): 16-byte cp.async copies spread over
  // all threads, each thread's copies completing as one arrival on xbar.  Weight stages:
  // every warp its first kStages (lane 0).  Zero / scale rows: every warp those of the
  // groups its own K range touches, with cp.async, awaited at first use (M <= 4: the end
  // of the first group segment); a group shared by two warps is copied by both (same
  // bytes).  Only the weight stages go through the TMA unit, which issues many small
  // copies slowly.
  {
    const int vecs = Kc / 8;                         // 16-byte vectors per token row
    for (int i = tid; i < Mc * vecs; i += kThreads) {
      const int m = i / vecs, v = i - m * vecs;
      cp_async16(sbase + off_xs + (uint32_t)(m * a.xs_stride + v * 8) * 2u,
                 a.x + (int64_t)(m0 + m) * a.ldx + krow0 + v * 8);
    }
    cp_async_arrive_noinc(xbar);
  }
  if (lane == 0) {
    for (int j = 0; j < kStages && j < nst; ++j) {
      sm100::mbar_arrive_expect_tx(full_bar(warp, j), kStageBytes);
      sm100::tma_load_2d(stage_addr(warp, j), &tmW, full_bar(warp, j), strip * 32,
                         (b0 + j * kBlocksPerStage) * 8);
    }
  }
  if (b1 > b0) {
    const int wg0 = b0 * 8 / a.gs - g0;              // this warp's first group row
    const int wgn = (b1 * 8 - 1) / a.gs - g0 - wg0 + 1;
    for (int i = lane; i < wgn * 40; i += 32) {
      const int gi = wg0 + i / 40, v = i % 40;      // 8 vectors of zeros, 32 of scales
      if (v < 8) {
        const int wc = strip * 32 + v * 4;
        if (wc < a.PN)
          cp_async16(sbase + off_zs + (uint32_t)(gi * 128 + v * 16),
                     a.qz + (int64_t)(g0 + gi) * a.PN + wc);
      } else {
        const int n = strip * kStripN + (v - 8) * 8;
        if (n < a.N)
          cp_async16(sbase + off_ss + (uint32_t)(gi * kStripN * 2 + (v - 8) * 16),
                     a.scales + (int64_t)(g0 + gi) * a.N + n);
      }
    }
  }
  bool ok = sm100::mbar_wait_bounded(xbar, 0, a.status);
  bool zs_ready = false;                             // this warp's zero / scale rows landed
  if (!BIAS) {
    cp_async_wait_all();
    __syncwarp();
    zs_ready = true;
  }

  const int chunk = (g >> 1) | ((g & 1) << 2);       // conflict-free word chunk
  float acc[TOKSETS][8][4];
#pragma unroll
  for (int s2 = 0; s2 < TOKSETS; ++s2)
#pragma unroll
    for (int q = 0; q < 8; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s2][q][i] = 0.f;

  int j = 0;                                          // stage counter of this warp
  {
    const uint32_t bsel = (g & 1) ? 0x1054u : 0x5410u;   // x into this lane's pair slot
    const uint32_t lane_off_a = (uint32_t)t * 128u + ((uint32_t)(chunk ^ t) << 4);
    const uint32_t lane_off_b = (uint32_t)(t + 4) * 128u + ((uint32_t)(chunk ^ (t + 4)) << 4);
    // shared-memory byte address of x[token][k = 0] for this lane's tokens (k is added
    // per block); a token beyond the chunk's Mc rows reads row 0 and is masked to zero
    uint32_t xrow[TOKSETS];
    uint32_t xmask[TOKSETS];
#pragma unroll
    for (int s2 = 0; s2 < TOKSETS; ++s2) {
      const int m = 4 * s2 + (g >> 1);
      const bool live = m < Mc;
      xmask[s2] = live ? 0xffffffffu : 0u;
      xrow[s2] = sbase + off_xs + (uint32_t)(((live ? m : 0) * a.xs_stride + t - krow0) * 2);
    }
    uint32_t zcst[4][4], scl[4][4];
    float pacc[BIAS ? 8 : 1][4];
    float gsc[BIAS ? 8 : 1][4];                         // M <= 4: the segment's scales
    for (int kb = b0 * 8; kb < b1 * 8 && ok;) {
      const int grp = kb / a.gs;
      const int kend = min(b1 * 8, (grp + 1) * a.gs);
      const int gl = grp - g0;
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
        // M <= 4: everything of the segment's zero / scale correction that does not need
        // the MMA results is done here, while the segment's stages are still in flight:
        // pacc starts at -(1024 + z) * sum(x) (resp. -(1024 + 16 z) * sum(x)), so after
        // the MMAs add sum((1024 + w) x) it holds sum((w - z) x) (resp. 16x that); the
        // scale (resp. scale / 16) is applied when the segment closes.
        if (!zs_ready) {
          cp_async_wait_all();
          __syncwarp();
          zs_ready = true;
        }
        float part = 0.f;                               // sum(x[token t]) over the segment
        if (t < Mc) {
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
        }
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        part += __shfl_xor_sync(0xffffffffu, part, 8);
        part += __shfl_xor_sync(0xffffffffu, part, 16);
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
            pacc[q][0] = -zl.x * part;
            pacc[q][1] = -zl.y * part;
            pacc[q][2] = -zh.x * part;
            pacc[q][3] = -zh.y * part;
            gsc[q][0] = sl.x;
            gsc[q][1] = sl.y;
            gsc[q][2] = sh.x * 0.0625f;
            gsc[q][3] = sh.y * 0.0625f;
          }
        }
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
            bf0[s2] = prmt(lds_u16(xa), 0u, bsel) & xmask[s2];
            bf1[s2] = prmt(lds_u16(xa + 8u), 0u, bsel) & xmask[s2];
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
        // close the group segment: apply the group's scale (the zero term is already in
        // pacc, seeded at the segment's start)
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[0][q][i] = fmaf(gsc[q][i], pacc[q][i], acc[0][q][i]);
      }
      kb = kend;
    }
  }
  if (!ok && lane == 0) {
    // a copy never arrived: wait (bounded) for this warp's copies still in flight
    for (int jj = j; jj < nst && jj < j + kStages; ++jj)
      sm100::mbar_wait_bounded(full_bar(warp, jj % kStages), (jj / kStages) & 1, nullptr,
                               50000000ull);
  }
  cp_async_wait_all();                               // no copy into this CTA outlives it
  __syncwarp();

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
  const size_t slot_stride = (size_t)MP * kStripN;
  // the tile's result leaves through emit(): fp16 to out, or (tensor parallel) fp32 to
  // this tile's slot on every rank for the fused all-reduce
  const bool ar = a.ar.world > 1;
  const uint32_t epoch = ar ? (uint32_t)*reinterpret_cast<volatile int*>(a.ar.state) : 0u;
  const uint32_t flag = epoch + 1u;
  const size_t ar_rank_stride = (size_t)a.ar.max_tiles * kArTileFloats;
  const size_t ar_tile = ((size_t)(epoch & 1u) * a.ar.world * a.ar.max_tiles + tile) * kArTileFloats;
  // fp32 sum plus the column's bias (when given), rounded once
  auto out_value = [&](int n, float v) {
    if (a.bias) v += __half2float(a.bias[n]);
    return __float2half_rn(v);
  };
  auto emit = [&](int idx, int m, int n, float v) {
    if (a.pair_strips > 0) {                           // parked for the SiLU-mul pair step
      a.pair_vals[(size_t)tile * slot_stride + idx] = a.bias ? v + __half2float(a.bias[n]) : v;
    } else if (!ar) {
      a.out[(int64_t)(m0 + m) * a.ldo + n] = out_value(n, v);
    } else {
      const size_t off = ar_tile + (size_t)a.ar.rank * ar_rank_stride + idx;
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r)
        if (r < a.ar.world) st_pair(a.ar.data[r] + off, v, flag);
    }
  };
  for (int idx = tid; idx < Mc * kStripN; idx += kThreads) {
    const int m = idx / kStripN, nl = idx - m * kStripN;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w)
      v += reinterpret_cast<const float*>(sgen + (uint32_t)w * kStages * kStageBytes)
               [m * DecGeo<TOKSETS>::kPartStride + nl];
    if (nsplit == 1) {
      const int n = nbase + nl;
      if (n < a.N) emit(idx, m, n, v);
    } else {
      a.part[(size_t)cta * slot_stride + idx] = v;
    }
  }
  if (nsplit > 1) {
    // ---- split-K: after the barrier, one thread takes a ticket with an acq_rel atomic
    // (gpu scope): its release is cumulative over the slot stores the barrier ordered
    // before it, its acquire (passed on by the next barrier) makes the other CTAs'
    // slots visible to the last CTA, which sums the tile's slots in slot order --------
    __syncthreads();
    if (tid == 0) *last_flag = (atom_add_acq_rel_gpu(a.cnt + tile, 1) == nsplit - 1) ? 1 : 0;
    __syncthreads();
    if (!*last_flag) return;
    for (int idx = tid; idx < Mc * kStripN; idx += kThreads) {
      const int m = idx / kStripN, nl = idx - m * kStripN;
      const int n = nbase + nl;
      if (n >= a.N) continue;
      const float* p = a.part + (size_t)first * slot_stride + idx;
      float v = 0.f;
      // 16 independent loads in flight together: one round trip to L2 for up to 16 slots
      for (int r0 = 0; r0 < nsplit; r0 += 16) {
        float v16[16];
#pragma unroll
        for (int r = 0; r < 16; ++r)
          v16[r] = (r0 + r < nsplit) ? __ldcg(p + (size_t)(r0 + r) * slot_stride) : 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r)
          if (r0 + r < nsplit) v += v16[r];            // slot order: deterministic
      }
      emit(idx, m, n, v);
    }
    if (tid == 0) a.cnt[tile] = 0;                     // ready for the next call
  }
  if (a.pair_strips > 0) {
    // ---- SiLU-mul pair step (same ticket protocol as split-K): the gate and up tiles of
    // one output strip are both final; the second to arrive rounds each to fp16, as the
    // product's output is rounded, and writes fp16(silu(g) * u) -------------------------
    const int s = strip, chunk_i = tile / a.strips;
    const bool up = s >= a.pair_strips;
    const int ps = up ? s - a.pair_strips : s;
    const int pid = chunk_i * a.pair_strips + ps;
    const int partner = chunk_i * a.strips + (up ? ps : ps + a.pair_strips);
    __syncthreads();
    if (tid == 0) *last_flag = (atom_add_acq_rel_gpu(a.pair_cnt + pid, 1) == 1) ? 1 : 0;
    __syncthreads();
    if (!*last_flag) return;
    const float* gv = a.pair_vals + (size_t)(up ? partner : tile) * slot_stride;
    const float* uv = a.pair_vals + (size_t)(up ? tile : partner) * slot_stride;
    const int nh = a.N / 2;
    for (int idx = tid; idx < Mc * kStripN; idx += kThreads) {
      const int m = idx / kStripN, nl = idx - m * kStripN;
      const int n = ps * kStripN + nl;
      if (n >= nh) continue;
      const float gg = __half2float(__float2half_rn(__ldcg(gv + idx)));
      const float uu = __half2float(__float2half_rn(__ldcg(uv + idx)));
      a.out[(int64_t)(m0 + m) * a.ldo + n] = __float2half_rn(gg * (1.0f / (1.0f + expf(-gg))) * uu);
    }
    if (tid == 0) a.pair_cnt[pid] = 0;
    return;
  }
  if (!ar) return;

  // ---- fused all-reduce of this tile (tensor parallel): every thread polls, in this
  // rank's buffer, the {value, flag} pairs of its own elements from every rank until the
  // flags read this call's number + 1 (bounded wait), then sums the values in rank order:
  // every rank computes the same bits ----------------------------------------------------
  {
    const unsigned long long* mine = a.ar.data[a.ar.rank] + ar_tile;
    bool late = false;
    for (int idx = tid; idx < Mc * kStripN; idx += kThreads) {
      const int m = idx / kStripN, nl = idx - m * kStripN;
      const int n = nbase + nl;
      if (n >= a.N) continue;
      float v = 0.f;
      for (int r = 0; r < a.ar.world; ++r) {
        const unsigned long long* p = mine + (size_t)r * ar_rank_stride + idx;
        uint2 e = ld_pair(p);
        if (e.y != flag && !late) {
          const uint64_t t0 = sm100::globaltimer_ns();
          for (uint32_t it = 0; e.y != flag; ++it) {
            e = ld_pair(p);
            if ((it & 63) == 63 && sm100::globaltimer_ns() - t0 > a.ar.timeout_ns) {
              atomicOr(a.status, kDevErrPeerTimeout);
              late = true;                             // no more waiting in this thread
              break;
            }
          }
        }
        v += __uint_as_float(e.x);                     // rank order
      }
      a.out[(int64_t)(m0 + m) * a.ldo + n] = out_value(n, v);
    }
  }
  __syncthreads();
  if (tid == 0) {
    // the call's last tile moves this rank to the next call number
    if (atomicAdd(a.ar.state + 1, 1) == a.strips * ((a.M + MP - 1) / MP) - 1) {
      a.ar.state[1] = 0;
      a.ar.state[0] += 1;
    }
  }
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

size_t smem_bytes(int xr, int xs_stride, int ngrp) {
  return 1024 + kRingBytes + kConsumers * kStages * 8 + 16 + 16 + (size_t)xr * xs_stride * 2 +
         (size_t)ngrp * (128 + kStripN * 2);
}

// Programmatic dependent launch is on unless AWQ_PDL=0 (read once per process): the
// next call's CTAs then become resident while this one streams, set up their barriers
// and warm L2 before the dependency is resolved.
bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AWQ_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int TOKSETS>
cudaError_t launch_t(const CUtensorMap& tm, const TmaGemvArgs& a, int grid, size_t smem,
                     cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  const cudaError_t attr = attr_once.run([] {
    return cudaFuncSetAttribute(gemv_tma_kernel<TOKSETS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvTmaMaxSmem);
  });
  if (attr != cudaSuccess) return attr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // programmatic dependent launch: the kernel waits (griddepcontrol.wait) before it
  // touches anything the previous grid may write
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<TOKSETS>, tm, a);
}

}  // namespace

// One CTA per SM when the tiles allow it (each CTA gets at least kMinStagesPerCta
// stages, a tile at most kMaxSplits CTAs and at most 64 / tokens); one more CTA per tile
// at a time while the largest K range's staged activations and zero / scale rows do not
// fit in shared memory.
bool plan_gemv_tma(int64_t M, int64_t N, int64_t K, int64_t gs, int num_sms, GemvTmaPlan* p) {
  if (M <= 0 || M > 16 || N <= 0 || N % 32 || gs % kRowsPerStage || K <= 0 || K % gs ||
      num_sms <= 0)
    return false;
  const int toksets = M <= 4 ? 1 : 2;
  const int64_t MP = 4 * toksets;
  const int64_t strips = (N + kStripN - 1) / kStripN;
  const int64_t tiles = strips * ((M + MP - 1) / MP);
  const int64_t nstage = K / kRowsPerStage;                   // stages per tile
  int64_t grid0 = tiles;
  if (tiles < num_sms) {
    // the last CTA of a tile reads (tokens x CTAs per tile) partial rows: keep it short
    const int64_t mc = M < MP ? M : MP;
    int64_t maxc = nstage / kMinStagesPerCta;
    if (maxc > kMaxSplits) maxc = kMaxSplits;
    if (maxc > 64 / mc) maxc = 64 / mc;
    if (maxc < 1) maxc = 1;
    grid0 = tiles * maxc < num_sms ? tiles * maxc : num_sms;
  }
  const int xr = toksets == 1 ? (int)M : 8;
  for (int64_t grid = grid0;; grid += tiles) {
    const int64_t b = grid / tiles, extra = grid % tiles;   // CTAs per tile: b or b + 1
    if (b > nstage || grid > 0x7fffffff) return false;
    const int64_t kc_max = (nstage + b - 1) / b * kRowsPerStage;   // rows of the largest range
    const int xs_stride = (int)kc_max + 8;                          // +16 B staggers token rows
    const int ngrp = (int)(kc_max / gs) + 2;
    const size_t smem = smem_bytes(xr, xs_stride, ngrp);
    if (smem > kGemvTmaMaxSmem) continue;
    const bool split = b > 1 || extra > 0;
    if (split && tiles > kMaxCounters) return false;
    p->toksets = toksets;
    p->strips = (int)strips;
    p->tiles = (int)tiles;
    p->grid = (int)grid;
    p->base = (int)b;
    p->extra = (int)extra;
    p->xr = xr;
    p->xs_stride = xs_stride;
    p->ngrp = ngrp;
    p->smem = smem;
    p->ws_bytes = split ? kCounterRegionBytes + (size_t)grid * MP * kStripN * sizeof(float) : 0;
    return true;
  }
}

// SiLU-mul epilogue: the gate and up halves must split at a strip boundary, and the tile
// and pair counters must fit the counter region.
bool gemv_tma_silu_ok(const GemvTmaPlan& p, int64_t N) {
  return N % (2 * kStripN) == 0 && p.strips % 2 == 0 &&
         (int64_t)p.tiles + p.tiles / 2 <= kMaxCounters;
}
size_t silu_vals_offset(const GemvTmaPlan& p) {
  return p.ws_bytes > 0 ? p.ws_bytes : kCounterRegionBytes;
}
size_t gemv_tma_silu_ws_bytes(const GemvTmaPlan& p) {
  const size_t mp = 4 * (size_t)p.toksets;
  return silu_vals_offset(p) + (size_t)p.tiles * mp * kStripN * sizeof(float);
}

bool gemv_tma_supported(const int32_t* qweight, int64_t N, int64_t ldx, const void* x) {
  return (N % 32 == 0) && ((reinterpret_cast<uintptr_t>(qweight) & 15) == 0) &&
         ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 8 == 0) && encode_fn() != nullptr;
}

cudaError_t launch_gemv_tma(const GemvTmaPlan& p, const void* x, int64_t ldx,
                            const int32_t* qweight, const int32_t* qzeros, const void* scales,
                            void* out, int64_t ldo, int M, int N, int K, int group_size,
                            void* workspace, int* dev_status, cudaStream_t stream,
                            const ArArgs* ar, const void* bias, bool silu_mul) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if ((p.ws_bytes > 0 || silu_mul) && !workspace) return cudaErrorInvalidValue;
  if (silu_mul && (!gemv_tma_silu_ok(p, N) || (ar && ar->world > 1))) return cudaErrorInvalidValue;
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)(N / 8), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)N / 2};
  cuuint32_t box[2] = {32, (cuuint32_t)kRowsPerStage};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          // 128-byte promotion, the size of one box row: 256 bytes measured 0.4 % slower
          // over the decode stack (1.1017 against 1.0976 ms per step)
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  TmaGemvArgs a;
  a.x = static_cast<const __half*>(x);
  a.ldx = ldx;
  a.qw = qweight;
  a.qz = qzeros;
  a.scales = static_cast<const __half*>(scales);
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.cnt = p.ws_bytes > 0 ? static_cast<int*>(workspace) : nullptr;
  a.part = p.ws_bytes > 0
               ? reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kCounterRegionBytes)
               : nullptr;
  a.M = M; a.N = N; a.K = K; a.gs = group_size; a.PN = N / 8; a.KB = K / 8;
  a.strips = p.strips;
  a.base = p.base;
  a.extra = p.extra;
  a.xs_stride = p.xs_stride;
  a.xr = p.xr;
  a.ngrp_cta = p.ngrp;
  a.l2pf = pdl_enabled() ? kL2PrefetchStages : 0;
  a.status = dev_status;
  a.bias = static_cast<const __half*>(bias);
  a.pair_strips = 0;
  a.pair_vals = nullptr;
  a.pair_cnt = nullptr;
  if (silu_mul) {
    // counters: split-K per tile at [0, tiles), pairs after them; values after the
    // split-K slots
    a.cnt = static_cast<int*>(workspace);
    a.pair_strips = p.strips / 2;
    a.pair_cnt = static_cast<int*>(workspace) + p.tiles;
    a.pair_vals = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) +
                                           silu_vals_offset(p));
  }
  if (ar) {
    a.ar = *ar;
  } else {
    a.ar = ArArgs{};
    a.ar.world = 1;
  }
  return p.toksets == 1 ? launch_t<1>(tm, a, p.grid, p.smem, stream)
                        : launch_t<2>(tm, a, p.grid, p.smem, stream);
}

}  // namespace awq
