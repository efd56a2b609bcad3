// awq_gemm_tc.cu -- AWQ W4A16 GEMMs on the sm_100a tensor cores (tcgen05 + TMEM): the
// prefill kernel (gemm_tc_kernel, below), the small-M kernel with the weights as the TMEM
// operand (gemm_ts_kernel, further down) and the split-K reduce kernel both use.
//
// Replaces _awq_gemm_kernel (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:152-228,
// 64x64 tiles on mma.sync) for M > 8.  The prefill kernel's CTA computes a 128 x 256 tile of
// out = x @ W with fp32 accumulation in tensor memory:
//
//   warp 0      TMA producer: per 64-deep K step loads the packed weight tile (64 rows
//               x 32 words), one row of scales (256 fp16) and one row of packed zeros
//               (32 words) into the weight ring (rfull[s]), and the x tile (128 or 256
//               x 64 fp16, 128-byte swizzle) into the x ring (afull[s]).  An x tile is
//               held until its MMAs complete, a weight tile only until it has been
//               dequantized, so the x ring is the deeper one: its depth x the K step
//               time must cover the load latency under load (~1.5 us) plus the
//               dequant and the MMAs
//   warps 2..9  dequant: int4 -> fp16 W tile, bit-exact (fp16 (w - z) * scale), one
//               8-row k-group per warp, written into the B ring as the UMMA B operand
//               in the MN-major 128-byte-swizzled canonical layout, then
//               fence.proxy.async + arrive on bfull[s] and rempty[s]; after the K loop
//               the same warps run the epilogue
//   warp 1      TMEM allocation (256 columns) and the single-thread MMA issue:
//               4 x tcgen05.mma.kind::f16 (M=128, N=256, K=16) per K step, then
//               tcgen05.commit -> aempty / bempty free the x and B stages; the last
//               commit signals the accumulator to the epilogue
//   epilogue    tcgen05.ld 32x32b (a warp reads its TMEM lane quarter = 32 rows, the
//               two warps of a quarter split the 256 columns), fp32 -> fp16, 16-byte
//               global stores (rows >= M / cols >= N masked)
//
// Shapes it takes (tc_supported): N % 32 == 0, group_size % 64 == 0 (so a K step
// lies in one group), ldx % 8 == 0 and 16-byte aligned pointers (TMA rules).
// Every mbarrier wait is bounded; a time-out sets the status word and the CTA
// drains its in-flight copies and MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "awq_common.cuh"
#include "awq_internal.h"
#include "awq_sm100.cuh"

namespace awq {

namespace {

constexpr int BN = 256, BK = 64;
constexpr int kDeqWarps = 8;                     // one 8-row k-group of a K step each
constexpr int kThreads = (2 + kDeqWarps) * 32;   // producer, MMA, dequant/epilogue
constexpr uint32_t B_BYTES = BN * BK * 2;        // 32 KB
constexpr uint32_t RAW_BYTES = BK * (BN / 8) * 4; // 8 KB
constexpr uint32_t SC_BYTES = BN * 2;             // 512 B
constexpr uint32_t ZR_BYTES = (BN / 8) * 4;       // 128 B
// B operand (MN-major, 128-byte swizzle): atom = 64 n x 8 k (1 KB); k-groups of 8
// are SBO = 1 KB apart, 64-wide n atoms LBO = 8 KB apart.
constexpr uint32_t B_SBO = 1024, B_LBO = 8 * 1024;
constexpr uint32_t A_SBO = 1024;                  // K-major: 8-row groups 1 KB apart
constexpr uint32_t kIdesc = sm100::idesc_f16_f32(128, BN, /*a_mn*/ 0, /*b_mn*/ 1);

// Tile geometry for NACC accumulators of 128 x 256 (BM = 128 * NACC rows per CTA).  Each
// dequantized B tile feeds NACC MMAs, so the dequant work per tensor flop falls as
// 1 / NACC.
template <int NACC>
struct Geo {
  static constexpr int BM = 128 * NACC;
  static constexpr int ASTAGES = NACC == 1 ? 5 : 4;   // x ring depth
  static constexpr int RSTAGES = NACC == 1 ? 4 : 3;   // packed weight / scale / zero ring
  static constexpr int BSTAGES = NACC == 1 ? 3 : 2;   // dequantized B ring depth
  static constexpr uint32_t A_BYTES = BM * BK * 2;    // 1 KB multiple (swizzle atoms)
  // every TMA destination starts on a 128-byte boundary: the SiLU-mul layout's second
  // (up) zero box goes to R_ZR + 128, not right after the first 64-byte box
  static constexpr uint32_t R_RAW = 0, R_SC = RAW_BYTES, R_ZR = R_SC + SC_BYTES;
  static constexpr uint32_t R_TX = RAW_BYTES + SC_BYTES + ZR_BYTES;
  static constexpr uint32_t R_STAGE = (R_ZR + 2 * 128 + 127) / 128 * 128;
  static_assert(R_SC % 128 == 0 && (R_SC + SC_BYTES / 2) % 128 == 0 && R_ZR % 128 == 0 &&
                    (RAW_BYTES / 2) % 128 == 0 && R_STAGE % 128 == 0,
                "TMA destinations 128-byte aligned");
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_R = OFF_A + ASTAGES * A_BYTES;
  static constexpr uint32_t OFF_B = (OFF_R + RSTAGES * R_STAGE + 1023) / 1024 * 1024;
  // afull, aempty, rfull, rempty, bfull, bempty, accf, tmem empty, drain
  static constexpr uint32_t OFF_BAR = OFF_B + BSTAGES * B_BYTES;
  static constexpr uint32_t NBARS = 2 * ASTAGES + 2 * RSTAGES + 2 * BSTAGES + 3;
  static constexpr uint32_t OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;      // + alignment slack
  static constexpr uint32_t TMEM_COLS = 256 * NACC;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

struct TcArgs {
  __half* out;
  int64_t ldo;
  int M, N, K, gs;
  int* status;
  const __half* bias;   // fp16 [N] added to every output row in fp32, or null
  int splits;           // CTAs along K per output tile (blockIdx.z); > 1: fp32 partials
  float* part;          // [splits][M][N] fp32 partials when splits > 1
  // stream-K (streamk != 0, splits == 1; tiles < gridDim.x): CTA c < tiles runs K steps
  // [0, sk_split) of tile c -- those CTAs move through K together, as one tile-per-CTA wave
  // does, so each x and weight slab is fetched from HBM once and read from L2 by the other
  // tiles of its row or column.  The other gridDim.x - tiles CTAs share the tiles' last
  // K/64 - sk_split steps evenly in linear (tile, step) order.  The last CTA to finish a
  // part of a tile sums the tile from fp32 slots.
  int streamk;
  int tiles_n;
  int sk_tiles;
  int sk_split;
  float* sk_part;       // [tiles][kSkSlots][BM * 256] fp32, each slot in fragment order
  int* sk_cnt;          // per-tile arrivals, zero between calls
  // persistent (streamk == 0, splits == 1; more tiles than CTAs): CTA c works on tiles
  // c, c + gridDim.x, ... of the tiles_m x tiles_n tiles (tile t = (t % tiles_m,
  // t / tiles_m), the order of the tile grid's blocks), one after another; the producer
  // loads the next tile's first stages while the epilogue writes the current one
  int persistent;
  int tiles_m;
  int tiles_total;
  // SiLU-mul epilogue (silu != 0; no split, no stream-K, no bias): columns [0, N/2) of the
  // weights are the gate, [N/2, N) the up projection.  Tile n's 256 B-operand columns are
  // gate columns [128 n, 128 n + 128) followed by the same up columns, loaded as two
  // half-width boxes each, and the epilogue writes out[m, 128 n + c] =
  // fp16(silu(g) * u) with g and u the fp16-rounded products (out is [M, N/2]).
  int silu;
};

// silu(g) * u of fp32 products rounded to fp16 first, as the unfused sequence rounds its
// product.  The sigmoid uses the hardware exponential and an approximate divide (two
// MUFU operations), as the reference's Triton sigmoid does (kernels/silu_mul.py:35-36):
// the epilogue runs while the tensor pipe waits for TMEM, and the IEEE forms cost ~10 us
// per 256 x 256 tile there.
__device__ __forceinline__ float silu_mul_rounded(float g, float u) {
  const float x = __half2float(__float2half_rn(g)), y = __half2float(__float2half_rn(u));
  return __fdividef(x, 1.0f + __expf(-x)) * y;
}

constexpr int kSkSlots = 3;   // CTAs per tile under stream-K, at most (the tail's sharers <= 2)
constexpr int kMaxSeg = 8;    // tiles a CTA works on under stream-K, at most

// One tile's part of a CTA's work: K steps [k0, k1) of tile (tile_m, tile_n), the idx-th
// of the n CTAs that work on the tile.
struct TcSeg {
  int tile_m, tile_n, k0, k1, idx, n;
};

// Writes one warp's 32 rows x 32 columns of fp16 results (`h`: this lane's row, 16 packed
// pairs) through 2 KB of shared memory at `stage`, so that each global store covers 8 rows
// x 64 contiguous bytes instead of 32 rows x 16 bytes.  The 16-byte chunks of a row are
// XOR-swizzled by (row / 2) % 4, which keeps both the row-wise writes and the chunk-wise
// reads free of bank conflicts.  Rows at or past M are not stored.
__device__ __forceinline__ void store_rows_staged(uint32_t stage, const uint32_t (&h)[16],
                                                  __half* out, int64_t ldo, int row0, int col,
                                                  int M, int lane) {
  const uint32_t sw = (uint32_t)(lane >> 1) & 3u;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    sm100::st_shared_v4(stage + (uint32_t)lane * 64u + (((uint32_t)j ^ sw) << 4), h[4 * j],
                        h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
  __syncwarp();
  const int ch = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const uint4 v = sm100::ld_shared_v4(stage + (uint32_t)r * 64u +
                                        (((uint32_t)ch ^ ((uint32_t)(r >> 1) & 3u)) << 4));
    if (row0 + r < M)
      *reinterpret_cast<uint4*>(out + (int64_t)(row0 + r) * ldo + col + ch * 8) = v;
  }
  __syncwarp();
}

// As store_rows_staged for 64 columns, so that each row segment a global store writes is
// one whole 128-byte line (col a multiple of 64 for that): stage_chunk64 writes this
// lane's row of 32-column chunk `part` (0 or 1) into 4 KB of shared memory at `stage`,
// flush_rows64 then writes the warp's 32 rows x 64 columns (columns at or past N, a
// multiple of 32, and rows at or past M are not stored).  The 16-byte chunks of a row are
// XOR-swizzled by row % 8, which keeps the row-wise writes and the chunk-wise reads free
// of bank conflicts.
__device__ __forceinline__ void stage_chunk64(uint32_t stage, const uint32_t (&h)[16], int part,
                                              int lane) {
  const uint32_t sw = (uint32_t)lane & 7u;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    sm100::st_shared_v4(stage + (uint32_t)lane * 128u + (((uint32_t)(4 * part + j) ^ sw) << 4),
                        h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
}
__device__ __forceinline__ void flush_rows64(uint32_t stage, __half* out, int64_t ldo, int row0,
                                             int col, int M, int N, int lane) {
  __syncwarp();
  const int ch = lane & 7;
  const bool col_ok = col + ch * 8 < N;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const uint4 v = sm100::ld_shared_v4(stage + (uint32_t)r * 128u +
                                        (((uint32_t)ch ^ ((uint32_t)r & 7u)) << 4));
    if (col_ok && row0 + r < M)
      *reinterpret_cast<uint4*>(out + (int64_t)(row0 + r) * ldo + col + ch * 8) = v;
  }
  __syncwarp();
}

__device__ __forceinline__ void epi_bar_sync() {       // the 8 dequant / epilogue warps
  asm volatile("bar.sync 1, %0;" ::"n"(kDeqWarps * 32) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <int NACC>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
               const TcArgs args) {
  using G = Geo<NACC>;
  constexpr int BM = G::BM, ASTAGES = G::ASTAGES, RSTAGES = G::RSTAGES, BSTAGES = G::BSTAGES;
  constexpr uint32_t A_BYTES = G::A_BYTES, R_STAGE = G::R_STAGE, R_RAW = G::R_RAW, R_SC = G::R_SC,
                     R_ZR = G::R_ZR, R_TX = G::R_TX;
  constexpr uint32_t OFF_A = G::OFF_A, OFF_R = G::OFF_R, OFF_B = G::OFF_B, OFF_BAR = G::OFF_BAR,
                     OFF_MISC = G::OFF_MISC;
  constexpr uint32_t TMEM_COLS = G::TMEM_COLS;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;        // 1 KB aligned (swizzle atoms)
  unsigned char* sgen = smem_raw + (sbase - base_raw);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // this CTA's work as segments (tile, K steps).  Tile grid: the tile of (blockIdx.x,
  // blockIdx.y), K steps split over blockIdx.z (the ranges of one tile differ by at most
  // one step).  Stream-K: CTA c < tiles takes steps [0, S) of tile c (slot 0); CTA
  // tiles + j of the G2 = gridDim.x - tiles others takes linear steps
  // [j TT / G2, (j + 1) TT / G2) of the tails, TT = tiles x L with L = K/64 - S, step u
  // being step S + u % L of tile u / L (slots 1 and 2 of a tile: its tail's first and
  // second sharer).  Persistent: tile blockIdx.x + i gridDim.x for segment i (seg_at).
  // The rings below count the CTA's steps from 0 across its segments.
  const int kt_all = args.K / BK;
  TcSeg seg[kMaxSeg];
  int nseg = 0;
  if (args.persistent) {
    nseg = (args.tiles_total - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  } else if (!args.streamk) {
    const int kt0 = (int)((int64_t)blockIdx.z * kt_all / args.splits);
    const int kt1 = (int)((int64_t)(blockIdx.z + 1) * kt_all / args.splits);
    seg[0] = TcSeg{(int)blockIdx.x, (int)blockIdx.y, kt0, kt1, (int)blockIdx.z, args.splits};
    nseg = 1;
  } else {
    const int T = args.sk_tiles, S = args.sk_split, L = kt_all - S;
    const int64_t G2 = (int64_t)gridDim.x - T, TT = (int64_t)T * L;
    auto start = [&](int64_t j) { return j * TT / G2; };
    auto cta_of = [&](int64_t u) {                    // the sharer whose range holds step u
      int64_t j = u * G2 / TT;
      if (j + 1 < G2 && start(j + 1) <= u) ++j;
      return j;
    };
    const int c = blockIdx.x;
    if (c < T) {
      const int64_t jf = cta_of((int64_t)c * L), jl = cta_of((int64_t)c * L + L - 1);
      seg[nseg++] = TcSeg{c / args.tiles_n, c % args.tiles_n, 0, S, 0, (int)(jl - jf) + 2};
    } else {
      const int64_t j = c - T, u1 = start(j + 1);
      int64_t u = start(j);
      for (; u < u1 && nseg < kMaxSeg;) {
        const int64_t t = u / L, tb = t * L;
        const int64_t e = u1 < tb + L ? u1 : tb + L;
        const int64_t jf = cta_of(tb), jl = cta_of(tb + L - 1);
        seg[nseg++] = TcSeg{(int)(t / args.tiles_n), (int)(t % args.tiles_n), S + (int)(u - tb),
                            S + (int)(e - tb), (int)(j - jf) + 1, (int)(jl - jf) + 2};
        u = e;
      }
      // the host keeps every share within kMaxSeg tiles and each tail within two sharers;
      // a launch outside that reports a shape error rather than drop steps
      if (u < u1 && tid == 0) atomicOr(args.status, kDevErrShape);
    }
    for (int si = 0; si < nseg; ++si)
      if (seg[si].n > kSkSlots) {
        if (tid == 0) atomicOr(args.status, kDevErrShape);
        nseg = 0;
      }
  }

  auto seg_at = [&](int si) -> TcSeg {
    if (args.persistent) {
      const int t = (int)blockIdx.x + si * (int)gridDim.x;
      return TcSeg{t % args.tiles_m, t / args.tiles_m, 0, kt_all, 0, 1};
    }
    return seg[si];
  };
  auto bar_afull = [&](int s) { return sbase + OFF_BAR + 8u * s; };
  auto bar_aempty = [&](int s) { return sbase + OFF_BAR + 8u * (ASTAGES + s); };
  auto bar_rfull = [&](int s) { return sbase + OFF_BAR + 8u * (2 * ASTAGES + s); };
  auto bar_rempty = [&](int s) { return sbase + OFF_BAR + 8u * (2 * ASTAGES + RSTAGES + s); };
  auto bar_bfull = [&](int s) { return sbase + OFF_BAR + 8u * (2 * ASTAGES + 2 * RSTAGES + s); };
  auto bar_bempty = [&](int s) {
    return sbase + OFF_BAR + 8u * (2 * ASTAGES + 2 * RSTAGES + BSTAGES + s);
  };
  const uint32_t bar_accf = sbase + OFF_BAR + 8u * (2 * ASTAGES + 2 * RSTAGES + 2 * BSTAGES);
  const uint32_t bar_tmem_empty = bar_accf + 8u;   // epilogue read the accumulator (stream-K)
  const uint32_t bar_drain = bar_accf + 16u;       // every MMA of this CTA completed
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sgen + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + OFF_MISC + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(sgen + OFF_MISC + 8);

  if (tid == 0) {
    for (int s = 0; s < ASTAGES; ++s) {
      sm100::mbar_init(bar_afull(s), 1);
      sm100::mbar_init(bar_aempty(s), 1);
    }
    for (int s = 0; s < RSTAGES; ++s) {
      sm100::mbar_init(bar_rfull(s), 1);
      sm100::mbar_init(bar_rempty(s), kDeqWarps);  // one arrive per dequant warp
    }
    for (int s = 0; s < BSTAGES; ++s) {
      sm100::mbar_init(bar_bfull(s), kDeqWarps);   // one arrive per dequant warp
      sm100::mbar_init(bar_bempty(s), 1);
    }
    sm100::mbar_init(bar_accf, 1);
    sm100::mbar_init(bar_tmem_empty, 1);
    sm100::mbar_init(bar_drain, 1);
    sm100::fence_mbar_init();
    *abort_flag = 0;
    sm100::prefetch_tmap(&tmA);
    sm100::prefetch_tmap(&tmW);
    sm100::prefetch_tmap(&tmS);
    sm100::prefetch_tmap(&tmZ);
  }
  if (warp == 1) {
    sm100::tmem_alloc(sbase + OFF_MISC, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer ----
    if (lane == 0) {
      // the CTA's step counter j is both rings' position; nr / na count the weight and
      // x stages issued (they differ by one when an abort falls between the two)
      int j = 0, nr = 0, na = 0;
      for (int si = 0; si < nseg && !*abort_flag; ++si) {
        const TcSeg sg = seg_at(si);
        for (int kt = sg.k0; kt < sg.k1; ++kt, ++j) {
          const int rs = j % RSTAGES, as = j % ASTAGES;
          const int k0 = kt * BK;
          const int grp = k0 / args.gs;
          if (j >= RSTAGES &&
              !sm100::mbar_wait_bounded(bar_rempty(rs), ((j / RSTAGES) & 1) ^ 1, args.status)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          const uint32_t rst = sbase + OFF_R + rs * R_STAGE;
          sm100::mbar_arrive_expect_tx(bar_rfull(rs), R_TX);
          if (!args.silu) {
            sm100::tma_load_2d(rst + R_RAW, &tmW, bar_rfull(rs), sg.tile_n * (BN / 8), k0);
            sm100::tma_load_2d(rst + R_SC, &tmS, bar_rfull(rs), sg.tile_n * BN, grp);
            sm100::tma_load_2d(rst + R_ZR, &tmZ, bar_rfull(rs), sg.tile_n * (BN / 8), grp);
          } else {
            // gate half, then up half: [64 rows][16 words] twice, 128 + 128 scales, 16 + 16
            // zero words (the maps' boxes are half as wide)
            const int hw = args.N / 16, hn = args.N / 2;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              sm100::tma_load_2d(rst + R_RAW + u * (RAW_BYTES / 2), &tmW, bar_rfull(rs),
                                 u * hw + sg.tile_n * (BN / 16), k0);
              sm100::tma_load_2d(rst + R_SC + u * (SC_BYTES / 2), &tmS, bar_rfull(rs),
                                 u * hn + sg.tile_n * (BN / 2), grp);
              sm100::tma_load_2d(rst + R_ZR + u * 128, &tmZ, bar_rfull(rs),
                                 u * hw + sg.tile_n * (BN / 16), grp);
            }
          }
          ++nr;
          if (j >= ASTAGES &&
              !sm100::mbar_wait_bounded(bar_aempty(as), ((j / ASTAGES) & 1) ^ 1, args.status)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          sm100::mbar_arrive_expect_tx(bar_afull(as), A_BYTES);
          sm100::tma_load_2d(sbase + OFF_A + as * A_BYTES, &tmA, bar_afull(as), k0, sg.tile_m * BM);
          ++na;
        }
      }
      // drain: the last (up to) RSTAGES weight and ASTAGES x copies must land before exit
      for (int i = (nr > RSTAGES ? nr - RSTAGES : 0); i < nr; ++i)
        sm100::mbar_wait_bounded(bar_rfull(i % RSTAGES), (i / RSTAGES) & 1, args.status);
      for (int i = (na > ASTAGES ? na - ASTAGES : 0); i < na; ++i)
        sm100::mbar_wait_bounded(bar_afull(i % ASTAGES), (i / ASTAGES) & 1, args.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer ------
    if (lane == 0) {
      int j = 0;
      for (int si = 0; si < nseg; ++si) {
        const TcSeg sg = seg_at(si);
        // a second segment reuses the accumulator: wait until the epilogue has read it
        if (si > 0) {
          if (!sm100::mbar_wait_bounded(bar_tmem_empty, (si - 1) & 1, args.status)) *abort_flag = 1;
          sm100::tc_fence_after();
        }
        for (int kt = sg.k0; kt < sg.k1 && !*abort_flag; ++kt, ++j) {
          const int as = j % ASTAGES, bs = j % BSTAGES;
          if (!sm100::mbar_wait_bounded(bar_bfull(bs), (j / BSTAGES) & 1, args.status) ||
              !sm100::mbar_wait_bounded(bar_afull(as), (j / ASTAGES) & 1, args.status)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          sm100::tc_fence_after();
          const uint32_t a0 = sbase + OFF_A + as * A_BYTES;
          const uint32_t b0 = sbase + OFF_B + bs * B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = sm100::umma_desc_sw128(b0 + kk * 2 * B_SBO, B_LBO, B_SBO);
#pragma unroll
            for (int h = 0; h < NACC; ++h) {   // rows [128 h, 128 h + 128) -> TMEM cols 256 h
              const uint64_t ad = sm100::umma_desc_sw128(a0 + h * 128 * 128 + kk * 32, 16, A_SBO);
              sm100::umma_f16(tmem_d + 256 * h, ad, bd, kIdesc, (kt != sg.k0 || kk != 0) ? 1u : 0u);
            }
          }
          sm100::umma_commit(bar_aempty(as));    // x tile consumed
          sm100::umma_commit(bar_bempty(bs));    // dequantized B consumed
        }
        sm100::umma_commit(bar_accf);            // phase si: the segment's MMAs have completed
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- dequant ---------
    const int dw = warp - 2;                 // 0..7: rows [8 dw, 8 dw + 8) of a K step
    const int w = lane;                      // packed word column within the tile
    const uint32_t bst_lane = (uint32_t)(w >> 3) * B_LBO + (uint32_t)dw * B_SBO;
    int j = 0;
    int pre = 0;                             // steps of this segment dequantized already
    for (int si = 0; si < nseg; ++si) {
      const TcSeg sg = seg_at(si);
      // The next segment's first step is dequantized before this segment's epilogue, so
      // that its MMAs can start as soon as the epilogue has read the accumulator (the
      // step body depends on the global step j only).
      const int extra = (si + 1 < nseg && seg_at(si + 1).k1 > seg_at(si + 1).k0) ? 1 : 0;
      for (int t = pre; t < (sg.k1 - sg.k0) + extra; ++t, ++j) {
        const int rs = j % RSTAGES, bs = j % BSTAGES;
        // The packed tile is dequantized into registers as soon as it lands and its weight
        // stage is released at once; only the shared-memory stores wait for the B stage
        // (freed by the MMAs of BSTAGES steps ago), so the dequant runs under the MMAs in
        // flight instead of between them.
        if (!sm100::mbar_wait_bounded(bar_rfull(rs), (j / RSTAGES) & 1, args.status)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const uint32_t rst = sbase + OFF_R + rs * R_STAGE;
        const uint32_t zw = sm100::ld_shared_u32(
            rst + R_ZR + (args.silu ? (uint32_t)(w >> 4) * 128u + 4u * (uint32_t)(w & 15) : 4u * (uint32_t)w));
        const uint4 s4 = sm100::ld_shared_v4(rst + R_SC + 16u * (uint32_t)w);
        uint32_t wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          // word w of row dw * 8 + i: one [64][32] block, or (SiLU-mul) the gate / up
          // [64][16] blocks for w < 16 / w >= 16
          const int r = dw * 8 + i;
          const uint32_t off = args.silu ? (uint32_t)(w >> 4) * (RAW_BYTES / 2) + 4u * (uint32_t)(r * 16 + (w & 15))
                                         : 4u * (uint32_t)(r * (BN / 8) + w);
          wv[i] = sm100::ld_shared_u32(rst + R_RAW + off);
        }
        uint32_t zc[4], sc[4] = {s4.x, s4.y, s4.z, s4.w};
        zero_consts(zw, zc);
        uint32_t d[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) dequant_word(wv[i], zc, sc, d[i]);
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(bar_rempty(rs));   // the warp's reads are done
        if (j >= BSTAGES &&
            !sm100::mbar_wait_bounded(bar_bempty(bs), ((j / BSTAGES) & 1) ^ 1, args.status)) {
          *abort_flag = 1;
          break;
        }
        const uint32_t bstage = sbase + OFF_B + bs * B_BYTES + bst_lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t addr = bstage + (uint32_t)i * 128u + ((uint32_t)((w & 7) ^ i) << 4);
          sm100::st_shared_v4(addr, d[i][0], d[i][1], d[i][2], d[i][3]);
        }
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(bar_bfull(bs));
      }
      pre = extra;

      // ----------------------------------------------------------- epilogue --------
      // the segment's accumulator: phase si of the accumulator barrier
      const bool ok = sm100::mbar_wait_bounded(bar_accf, si & 1, args.status);
      sm100::tc_fence_after();
      const int q = warp & 3;                  // TMEM lane quarter this warp may access
      const int half = dw >> 2;                // the two warps of a quarter split the work
      // NACC == 1: split the 256 columns; NACC == 2: one accumulator (128 rows) each
      const int acc = NACC == 2 ? half : 0;
      const int c_lo = NACC == 2 ? 0 : half * 4, c_hi = NACC == 2 ? 8 : half * 4 + 4;
      const int rloc = acc * 128 + q * 32 + lane;   // row within the tile
      const int row = sg.tile_m * BM + rloc;
      const uint32_t taddr = tmem_d + acc * 256 + ((uint32_t)(q * 32) << 16);
      // stream-K: a tile shared by several CTAs leaves this CTA as an fp32 partial in the
      // tile's slot sg.idx; the last CTA to arrive sums the slots
      const bool shared_tile = args.streamk && sg.n > 1;
      const int tile = sg.tile_m * args.tiles_n + sg.tile_n;
      float* slot = shared_tile ? args.sk_part + ((size_t)tile * kSkSlots + sg.idx) * BM * BN
                                : nullptr;
      // fp16 results leave through 4 KB of shared memory per warp in B stage j % BSTAGES:
      // every MMA of this segment has completed (the accumulator barrier), and the stage
      // that holds the next segment's first step, if any, is (j - 1) % BSTAGES
      static_assert(kDeqWarps * 4096 <= B_BYTES, "epilogue staging fits in one B stage");
      const uint32_t stage = sbase + OFF_B + (uint32_t)(j % BSTAGES) * B_BYTES + (uint32_t)dw * 4096u;
      const int row0 = sg.tile_m * BM + acc * 128 + q * 32;
      const bool live = ok && !*abort_flag;
      if (!shared_tile && args.silu) {
        // gate chunk cg (TMEM columns 32 cg) with up chunk cg + 4 (columns 128 + 32 cg):
        // NACC == 2: chunks 0..3 of this warp's accumulator; NACC == 1: the warp's half
        const int g_lo = NACC == 2 ? 0 : half * 2, g_hi = NACC == 2 ? 4 : half * 2 + 2;
        // one 32-column chunk per store (pairing two chunks per 128-byte line, as the plain
        // output does, made this path slower: gate+up at M = 2048 443 us against 424)
        if (live) {
#pragma unroll 1
          for (int cg = g_lo; cg < g_hi; ++cg) {
            uint32_t vg[32], vu[32];
            sm100::tmem_ld_32x32b_x32(taddr + cg * 32, vg);
            sm100::tmem_ld_32x32b_x32(taddr + 128 + cg * 32, vu);
            sm100::tmem_ld_wait();
            const int col = sg.tile_n * (BN / 2) + cg * 32;
            uint32_t h[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              h[jj] = h2_as_u32(__floats2half2_rn(
                  silu_mul_rounded(__uint_as_float(vg[2 * jj]), __uint_as_float(vu[2 * jj])),
                  silu_mul_rounded(__uint_as_float(vg[2 * jj + 1]), __uint_as_float(vu[2 * jj + 1]))));
            store_rows_staged(stage, h, args.out, args.ldo, row0, col, args.M, lane);
          }
        }
      } else if (!shared_tile && args.splits == 1) {
        // fp16 output, two 32-column chunks per store (whole 128-byte lines per row; the
        // chunk count, 8 or 4, is even)
        if (live) {
#pragma unroll 1
          for (int c = c_lo; c < c_hi; c += 2) {
            const int col = sg.tile_n * BN + c * 32;
            if (col >= args.N) continue;         // the same for the whole warp
#pragma unroll 1
            for (int part = 0; part < 2; ++part) {
              uint32_t v[32];
              sm100::tmem_ld_32x32b_x32(taddr + (c + part) * 32, v);
              sm100::tmem_ld_wait();
              const int ccol = col + part * 32;
              if (args.bias && ccol < args.N) {  // the columns' bias, added in fp32
#pragma unroll
                for (int jj = 0; jj < 32; ++jj)
                  v[jj] = __float_as_uint(__uint_as_float(v[jj]) + __half2float(args.bias[ccol + jj]));
              }
              uint32_t h[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                h[jj] = h2_as_u32(__floats2half2_rn(__uint_as_float(v[2 * jj]), __uint_as_float(v[2 * jj + 1])));
              stage_chunk64(stage, h, part, lane);
            }
            flush_rows64(stage, args.out, args.ldo, row0, col, args.M, args.N, lane);
          }
        }
      } else if (!shared_tile) {
        if (live) {
#pragma unroll 1
          for (int c = c_lo; c < c_hi; ++c) {
            uint32_t v[32];
            sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
            sm100::tmem_ld_wait();
            const int col = sg.tile_n * BN + c * 32;
            if (col >= args.N) continue;         // the same for the whole warp
            if (args.splits > 1) {
              // the split-K plane, summed with the bias by the reduce kernel
              if (row >= args.M) continue;
              float4* dst = reinterpret_cast<float4*>(
                  args.part + ((size_t)blockIdx.z * args.M + row) * args.N + col);
#pragma unroll
              for (int jj = 0; jj < 8; ++jj)
                dst[jj] = make_float4(__uint_as_float(v[4 * jj]), __uint_as_float(v[4 * jj + 1]),
                                      __uint_as_float(v[4 * jj + 2]), __uint_as_float(v[4 * jj + 3]));
            } else {
              if (args.bias) {                  // the columns' bias, added in fp32
#pragma unroll
                for (int jj = 0; jj < 32; ++jj)
                  v[jj] = __float_as_uint(__uint_as_float(v[jj]) + __half2float(args.bias[col + jj]));
              }
              uint32_t h[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                h[jj] = h2_as_u32(__floats2half2_rn(__uint_as_float(v[2 * jj]), __uint_as_float(v[2 * jj + 1])));
              store_rows_staged(stage, h, args.out, args.ldo, row0, col, args.M, lane);
            }
          }
        }
      } else {
        // A part of a shared tile.  If the tile's other n - 1 parts are already in their
        // slots (an acquire load of the tile's counter), this CTA sums the tile at once and
        // never writes its own slot.  Otherwise it writes its slot (fp32, fragment order:
        // float4 (c * 8 + jj) of row rloc at (c * 8 + jj) * BM + rloc, so a warp's store
        // covers 512 contiguous bytes) and takes a ticket (acq_rel, gpu scope; its release
        // covers the slot stores the barrier ordered before it); the last ticket sums.  The
        // sum runs in slot order -- the same bits whichever CTA makes it -- with this CTA's
        // own part read back from TMEM, then adds the bias, writes fp16 and clears the
        // counter for the next call.
        if (dw == 0 && lane == 0) *last_flag = ld_acquire_gpu(args.sk_cnt + tile) == sg.n - 1 ? 1 : 0;
        epi_bar_sync();
        if (!*last_flag) {
          if (live) {
#pragma unroll 1
            for (int c = c_lo; c < c_hi; ++c) {
              uint32_t v[32];
              sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
              sm100::tmem_ld_wait();
              float4* dst = reinterpret_cast<float4*>(slot) + (size_t)c * 8 * BM + rloc;
#pragma unroll
              for (int jj = 0; jj < 8; ++jj)
                dst[(size_t)jj * BM] = make_float4(__uint_as_float(v[4 * jj]), __uint_as_float(v[4 * jj + 1]),
                                                   __uint_as_float(v[4 * jj + 2]), __uint_as_float(v[4 * jj + 3]));
            }
          }
          epi_bar_sync();
          if (dw == 0 && lane == 0)
            *last_flag = (atom_add_acq_rel_gpu(args.sk_cnt + tile, 1) == sg.n - 1) ? 1 : 0;
          epi_bar_sync();
        }
        if (*last_flag) {
          if (live) {
            // the other parts' slots: o0 < o1 (o1 < 0 when the tile has two parts).  Each
            // round has 16 float4 loads per thread in flight: two chunks of the one other
            // slot, or one chunk of both.
            const int o0 = sg.idx == 0 ? 1 : 0;
            const int o1 = sg.n < 3 ? -1 : (sg.idx == 2 ? 1 : 2);
            const bool two = o1 < 0;
            const float4* tbase =
                reinterpret_cast<const float4*>(args.sk_part + (size_t)tile * kSkSlots * BM * BN) + rloc;
#pragma unroll 1
            for (int c = c_lo; c < c_hi; c += two ? 2 : 1) {
              const float4* s0 = tbase + (size_t)o0 * (BM * BN / 4) + (size_t)c * 8 * BM;
              const float4* s1 = two ? s0 + (size_t)8 * BM
                                     : tbase + (size_t)o1 * (BM * BN / 4) + (size_t)c * 8 * BM;
              float4 p0[8], p1[8];
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                p0[jj] = __ldcg(s0 + (size_t)jj * BM);
                p1[jj] = __ldcg(s1 + (size_t)jj * BM);
              }
#pragma unroll 1
              for (int k = 0; k < (two ? 2 : 1); ++k) {
                const int cc = c + k;
                const int col = sg.tile_n * BN + cc * 32;
                if (col >= args.N) continue;     // the same for the whole warp
                uint32_t v[32];
                sm100::tmem_ld_32x32b_x32(taddr + cc * 32, v);
                sm100::tmem_ld_wait();
                float sum[32];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const float4 f0 = (two && k == 1) ? p1[jj] : p0[jj];
                  const float4 f1 = p1[jj];
                  const float own[4] = {__uint_as_float(v[4 * jj]), __uint_as_float(v[4 * jj + 1]),
                                        __uint_as_float(v[4 * jj + 2]), __uint_as_float(v[4 * jj + 3])};
                  const float a0[4] = {f0.x, f0.y, f0.z, f0.w}, a1[4] = {f1.x, f1.y, f1.z, f1.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    // parts in slot order 0, 1, 2 from 0.0f: own part at sg.idx, then the
                    // other slots o0 (a0) and o1 (a1) in their places
                    float acc = 0.f;
                    acc += sg.idx == 0 ? own[e] : a0[e];
                    acc += sg.idx == 1 ? own[e] : (sg.idx == 0 ? a0[e] : a1[e]);
                    if (!two) acc += sg.idx == 2 ? own[e] : a1[e];
                    sum[4 * jj + e] = acc;
                  }
                }
                if (args.bias) {
#pragma unroll
                  for (int jj = 0; jj < 32; ++jj) sum[jj] += __half2float(args.bias[col + jj]);
                }
                uint32_t h[16];
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) h[jj] = h2_as_u32(__floats2half2_rn(sum[2 * jj], sum[2 * jj + 1]));
                store_rows_staged(stage, h, args.out, args.ldo, row0, col, args.M, lane);
              }
            }
          }
          if (dw == 0 && lane == 0) args.sk_cnt[tile] = 0;   // ready for the next call
        }
      }
      // every epilogue thread has read the accumulator and left the staging area (the B
      // stage that the next segment's second step is dequantized into)
      sm100::tc_fence_before();
      epi_bar_sync();
      if (si + 1 < nseg && dw == 0 && lane == 0) sm100::mbar_arrive(bar_tmem_empty);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    // every MMA this CTA issued has completed (in the abort path some may still be in
    // flight) before the columns go back: one more commit, bounded wait
    if (lane == 0) {
      sm100::umma_commit(bar_drain);
      sm100::mbar_wait_bounded(bar_drain, 0, nullptr, 100000000ull);
    }
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_d, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// Small-M kernel (M <= 64): the dequantized weights are the TMEM operand.
//
// out^T = W^T x^T: the tensor core's M dimension is 128 output columns (TMEM lanes),
// its N dimension the NT tokens of the tile, so the MMA work shrinks with the token
// count.  The dequant warps write W straight into tensor memory with tcgen05.st, so the
// dequantized tile never passes through shared memory.  Per CTA: 256 columns x NT
// tokens, K steps of 64 rows.
//
//   warp 0      TMA: x tile (NT x 64 fp16, 128-byte swizzle), packed weight tile (64 x 32
//               words, 128-byte swizzle), one scale row, one zero row -> ring of TSTAGES
//   warps 2..9  dequant into TMEM stage `as` (64 columns: two 128-lane halves x 32
//               columns of k pairs); warp w owns lane quarter q = w % 4 and K blocks
//               {2r, 2r+1} of the step, r = (w - 2) / 4
//   warp 1      MMA: per step 2 halves x 4 K blocks of tcgen05.mma (M = 128, N = NT,
//               K = 16, A from TMEM, B = x from shared memory); one commit per step
//               frees both rings
//   epilogue    tcgen05.ld 32x32b: thread = one output column, NT tokens
//
// What bounds it (measured on B200): a tcgen05.mma of this shape costs ~30 ns however
// small N is (one of M = 128, N = 256, K = 16 costs ~71 ns), and each covers only 2048
// weights, so the 8 MMAs of a K step take ~240 ns -- about the time HBM needs for the
// step's 8.6 KB per SM.  With the per-step handshakes the kernel runs at ~0.5-0.7 of HBM
// speed whatever NT is: slower than the mma.sync decode kernel up to 8 tokens, faster
// than it (which re-reads the weights per 8 tokens) and than the prefill kernel's split
// from 9 to 64 tokens on the shapes that need a K split (output dispatch in awq_capi.cu).
//
// Lane map.  In quarter q the thread (t0, t1) = (t % 4, t / 4) of a dequant warp holds
// packed word column wc = 8 q + t1 of the tile and k rows 16 r + 4 t0 .. + 3 of each K
// block (the tcgen05.st 16x256b fragment gives it columns 2 t0, 2 t0 + 1, i.e. those k
// pairs).  Its 8 output slots are the 8 nibble slots u of the word: slot u goes to half
// h = u / 4, lane 32 q + 8 (u % 4) + t1, and is element [0,2,4,6,1,3,5,7][u] of the word.
// Lanes, halves and output columns map one to one; the epilogue inverts the map.
//
// SiLU-mul mode (args.silu): packed words 0-15 of the tile are gate words, 16-31 the
// matching up words, so lane quarter q + 2 holds the up column of quarter q's gate column
// in the same lane and half; the epilogue pairs them through shared memory.
constexpr int kTsAStages = 4;                   // TMEM A stages of 64 columns
constexpr uint32_t kTsTmemCols = 512;
constexpr uint32_t kTsDCol = kTsAStages * 64;    // accumulators: 2 halves x NT columns
constexpr int kTsMinSteps = 4;                   // K steps per CTA at least (split-K)

template <int NT>
struct TsGeo {
  static constexpr uint32_t X_BYTES = NT * BK * 2;
  static constexpr uint32_t T_RAW = X_BYTES;     // 1 KB multiple (swizzle atoms)
  static constexpr uint32_t T_SC = T_RAW + RAW_BYTES, T_ZR = T_SC + SC_BYTES;
  static constexpr uint32_t T_STAGE = (T_ZR + ZR_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t TX_BYTES = X_BYTES + RAW_BYTES + SC_BYTES + ZR_BYTES;
  static constexpr int TSTAGES = (200 * 1024) / T_STAGE < 16 ? (200 * 1024) / T_STAGE : 16;
  static constexpr uint32_t OFF_BAR = TSTAGES * T_STAGE;
  static constexpr uint32_t NBARS = 2 * TSTAGES + kTsAStages + 1;   // tfull, tempty, afull, accf
  static constexpr uint32_t OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(X_BYTES % 1024 == 0, "x tile must keep the weight tile 1 KB aligned");
  // SiLU-mul mode: every TMA destination 128-byte aligned (the up half of the weight tile
  // at T_RAW + 4 KB, of the scales at T_SC + 256, of the zeros at T_ZR + 128)
  static_assert(T_SC % 128 == 0 && T_ZR % 128 == 0 && T_ZR + 128 + ZR_BYTES / 2 <= T_STAGE,
                "SiLU-mul half boxes");
  static_assert(NT * 128 * 4 <= TSTAGES * T_STAGE, "SiLU-mul epilogue exchange");
  static_assert(kTsDCol + 2 * NT <= kTsTmemCols, "TMEM columns");
  static_assert(TSTAGES >= kTsAStages, "the copy-stage barriers also free the TMEM A stages");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_ts_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
               const TcArgs args) {
  using G = TsGeo<NT>;
  constexpr int TSTAGES = G::TSTAGES, ASTAGES = kTsAStages;
  constexpr uint32_t T_STAGE = G::T_STAGE, T_RAW = G::T_RAW, T_SC = G::T_SC, T_ZR = G::T_ZR;
  constexpr uint32_t OFF_BAR = G::OFF_BAR, OFF_MISC = G::OFF_MISC, TX_BYTES = G::TX_BYTES;
  constexpr uint32_t kIdescTs = sm100::idesc_f16_f32(128, NT, /*a_mn*/ 0, /*b_mn*/ 0);
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base_raw = sm100::smem_u32(smem_raw);
  const uint32_t sbase = (base_raw + 1023u) & ~1023u;
  unsigned char* sgen = smem_raw + (sbase - base_raw);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int tile_m = blockIdx.x, tile_n = blockIdx.y;
  const int kt_all = args.K / BK;
  const int kt0 = (int)((int64_t)blockIdx.z * kt_all / args.splits);
  const int KT = (int)((int64_t)(blockIdx.z + 1) * kt_all / args.splits) - kt0;

  auto bar_tfull = [&](int s) { return sbase + OFF_BAR + 8u * s; };
  auto bar_tempty = [&](int s) { return sbase + OFF_BAR + 8u * (TSTAGES + s); };
  auto bar_afull = [&](int s) { return sbase + OFF_BAR + 8u * (2 * TSTAGES + s); };
  const uint32_t bar_accf = sbase + OFF_BAR + 8u * (2 * TSTAGES + ASTAGES);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sgen + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + OFF_MISC + 4);

  if (tid == 0) {
    for (int s = 0; s < TSTAGES; ++s) {
      sm100::mbar_init(bar_tfull(s), 1);
      sm100::mbar_init(bar_tempty(s), 1);
    }
    for (int s = 0; s < ASTAGES; ++s) sm100::mbar_init(bar_afull(s), kDeqWarps);
    sm100::mbar_init(bar_accf, 1);
    sm100::fence_mbar_init();
    *abort_flag = 0;
    sm100::prefetch_tmap(&tmX);
    sm100::prefetch_tmap(&tmW);
    sm100::prefetch_tmap(&tmS);
    sm100::prefetch_tmap(&tmZ);
  }
  if (warp == 1) {
    sm100::tmem_alloc(sbase + OFF_MISC, kTsTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer ----
    if (lane == 0) {
      int kt = 0;
      for (; kt < KT; ++kt) {
        const int s = kt % TSTAGES;
        if (kt >= TSTAGES &&
            !sm100::mbar_wait_bounded(bar_tempty(s), ((kt / TSTAGES) & 1) ^ 1, args.status)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int k0 = (kt0 + kt) * BK;
        const int grp = k0 / args.gs;
        const uint32_t st = sbase + s * T_STAGE;
        sm100::mbar_arrive_expect_tx(bar_tfull(s), TX_BYTES);
        sm100::tma_load_2d(st, &tmX, bar_tfull(s), k0, tile_m * NT);
        if (args.silu) {
          // gate words [16 n, 16 n + 16) and the same up words, N / 16 further on
          const int gw = tile_n * (BN / 16), uw = args.N / 16 + gw;
          sm100::tma_load_2d(st + T_RAW, &tmW, bar_tfull(s), gw, k0);
          sm100::tma_load_2d(st + T_RAW + RAW_BYTES / 2, &tmW, bar_tfull(s), uw, k0);
          sm100::tma_load_2d(st + T_SC, &tmS, bar_tfull(s), gw * 8, grp);
          sm100::tma_load_2d(st + T_SC + SC_BYTES / 2, &tmS, bar_tfull(s), uw * 8, grp);
          sm100::tma_load_2d(st + T_ZR, &tmZ, bar_tfull(s), gw, grp);
          sm100::tma_load_2d(st + T_ZR + 128, &tmZ, bar_tfull(s), uw, grp);
        } else {
          sm100::tma_load_2d(st + T_RAW, &tmW, bar_tfull(s), tile_n * (BN / 8), k0);
          sm100::tma_load_2d(st + T_SC, &tmS, bar_tfull(s), tile_n * BN, grp);
          sm100::tma_load_2d(st + T_ZR, &tmZ, bar_tfull(s), tile_n * (BN / 8), grp);
        }
      }
      for (int j = (kt > TSTAGES ? kt - TSTAGES : 0); j < kt; ++j)
        sm100::mbar_wait_bounded(bar_tfull(j % TSTAGES), (j / TSTAGES) & 1, args.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer ------
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int ts = kt % TSTAGES, as = kt % ASTAGES;
        if (!sm100::mbar_wait_bounded(bar_afull(as), (kt / ASTAGES) & 1, args.status)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        sm100::tc_fence_after();
        const uint32_t x0 = sbase + ts * T_STAGE;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bd = sm100::umma_desc_sw128(x0 + kk * 32, 16, A_SBO);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            sm100::umma_f16_ts(tmem + kTsDCol + h * NT, tmem + as * 64 + h * 32 + kk * 8, bd,
                               kIdescTs, (kt | kk) != 0);
        }
        // one commit frees both the copy stage and the TMEM A stage of this step
        sm100::umma_commit(bar_tempty(ts));
      }
      sm100::umma_commit(bar_accf);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- dequant ---------
    const int q = warp & 3;                  // TMEM lane quarter of this warp
    const int rb = ((warp - 2) >> 2) * 2;    // first of its two 16-row K blocks
    const int t0 = lane & 3, t1 = lane >> 2;
    const int wc = 8 * q + t1;               // packed word column within the tile
    // Byte offsets of this thread's 8 packed words of a K step within the weight tile.
    // One 32-word box: 128-byte rows, 128-byte swizzle (16-byte chunk ^= row % 8).
    // SiLU-mul: two 16-word boxes (gate, then up 4 KB further), 64-byte rows, 64-byte
    // swizzle (16-byte chunk ^= (row / 2) % 4).
    uint32_t woff[2][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t row = 16 * (rb + rr) + 4 * t0 + i;
        woff[rr][i] = args.silu
                          ? (uint32_t)(wc >> 4) * (RAW_BYTES / 2) + row * 64 +
                                ((((uint32_t)(wc & 15) >> 2) ^ ((row >> 1) & 3)) << 4) +
                                ((uint32_t)(wc & 3) << 2)
                          : row * 128 + (((uint32_t)(wc >> 2) ^ (row & 7)) << 4) +
                                ((uint32_t)(wc & 3) << 2);
      }
    const uint32_t zoff = args.silu ? (uint32_t)(wc >> 4) * 128u + 4u * (uint32_t)(wc & 15)
                                    : 4u * (uint32_t)wc;
    uint32_t zc[8], sc[8];
    int grp_have = -1;
    for (int kt = 0; kt < KT; ++kt) {
      const int ts = kt % TSTAGES, as = kt % ASTAGES;
      if (!sm100::mbar_wait_bounded(bar_tfull(ts), (kt / TSTAGES) & 1, args.status)) {
        *abort_flag = 1;
        break;
      }
      // TMEM A stage `as` is free once the MMAs of step j = kt - ASTAGES have completed,
      // which the copy-stage barrier of step j records (phase j / TSTAGES of slot
      // j % TSTAGES; TSTAGES >= ASTAGES, and that slot cannot complete step j + TSTAGES
      // before this warp has dequantized step kt, so the parity cannot alias)
      if (kt >= ASTAGES) {
        const int j = kt - ASTAGES;
        if (!sm100::mbar_wait_bounded(bar_tempty(j % TSTAGES), (j / TSTAGES) & 1, args.status)) {
          *abort_flag = 1;
          break;
        }
      }
      if (*abort_flag) break;
      sm100::tc_fence_after();
      const unsigned char* tst = sgen + ts * T_STAGE;
      const int grp = (kt0 + kt) * BK / args.gs;
      if (grp != grp_have) {
        grp_have = grp;
        const uint32_t zw = *reinterpret_cast<const uint32_t*>(tst + T_ZR + zoff);
        const uint4 s4 = reinterpret_cast<const uint4*>(tst + T_SC)[wc];
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t zb = __byte_perm(zw, zw, 0x1111u * (uint32_t)b);
          zc[2 * b] = lop3_and_or(zb, kLoMask, kMagic);                              // 1024 + z
          zc[2 * b + 1] = hmul2_u32(lop3_and_or(zb, kHiMask, kMagic), kNegInv16);    // -(64 + z)
        }
        // slot u holds element [0,2,4,6,1,3,5,7][u]: scale half (u / 4) of word u % 4
#pragma unroll
        for (int u = 0; u < 8; ++u) sc[u] = __byte_perm(sw[u & 3], sw[u & 3], u < 4 ? 0x1010u : 0x3232u);
      }
      const uint32_t raw = sbase + ts * T_STAGE + T_RAW;
      uint32_t o[2][8][2];                   // [K block][slot][k pair]
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        uint32_t a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          asm volatile("ld.shared.b32 %0, [%1];" : "=r"(a[i]) : "r"(raw + woff[rr][i]));
#pragma unroll
        for (int p = 0; p < 2; ++p) {
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            // byte b of row 2p -> bytes 0, 1; byte b of row 2p + 1 -> bytes 2, 3: the k pair
            // (low half: row 2p) of slots 2b (low nibbles) and 2b + 1 (high nibbles)
            const uint32_t xb = __byte_perm(a[2 * p], a[2 * p + 1], 0x4400u + 0x1111u * (uint32_t)b);
            o[rr][2 * b][p] =
                hmul2_u32(hsub2_u32(lop3_and_or(xb, kLoMask, kMagic), zc[2 * b]), sc[2 * b]);
            o[rr][2 * b + 1][p] = hmul2_u32(
                hfma2_u32(lop3_and_or(xb, kHiMask, kMagic), kInv16, zc[2 * b + 1]), sc[2 * b + 1]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int lb = 0; lb < 2; ++lb) {
          const int u0 = 4 * h + 2 * lb, u1 = u0 + 1;
          const uint32_t r8[8] = {o[0][u0][0], o[0][u0][1], o[0][u1][0], o[0][u1][1],
                                  o[1][u0][0], o[1][u0][1], o[1][u1][0], o[1][u1][1]};
          const uint32_t taddr =
              tmem + ((uint32_t)(32 * q + 16 * lb) << 16) + as * 64 + h * 32 + rb * 8;
          sm100::tmem_st_16x256b_x2(taddr, r8);
        }
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(bar_afull(as));
    }

    // ------------------------------------------------------------- epilogue --------
    const bool ok = sm100::mbar_wait_bounded(bar_accf, 0, args.status);
    sm100::tc_fence_after();
    if (args.silu) {
      // Lane quarters 2 and 3 hold the up columns of the gate columns in quarters 0 and 1
      // (same lane, same half): they pass their fp32 sums through the ring's shared memory
      // (every copy has landed and every MMA has read its operands once the accumulators
      // are complete), laid out [token][column]; quarters 0 and 1 write
      // out[m, 128 n + c] = fp16(silu(g) * u).  Every dequant warp meets the barrier once.
      const bool go = ok && !*abort_flag;
      const int h = (warp - 2) >> 2;
      const int u = 4 * h + (lane >> 3);
      const int e = u < 4 ? 2 * u : 2 * (u - 4) + 1;
      const int cl = 8 * (8 * (q & 1) + (lane & 7)) + e;   // column among the tile's 128
      float* xch = reinterpret_cast<float*>(sgen);
      if (go && q >= 2) {
#pragma unroll
        for (int c = 0; c < NT / 16; ++c) {
          uint32_t v[16];
          sm100::tmem_ld_32x32b_x16(tmem + ((uint32_t)(32 * q) << 16) + kTsDCol + h * NT + c * 16, v);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) xch[(c * 16 + j) * 128 + cl] = __uint_as_float(v[j]);
        }
      }
      epi_bar_sync();
      if (go && q < 2) {
        __half* dst = args.out + (int64_t)tile_n * (BN / 2) + cl;
#pragma unroll
        for (int c = 0; c < NT / 16; ++c) {
          uint32_t v[16];
          sm100::tmem_ld_32x32b_x16(tmem + ((uint32_t)(32 * q) << 16) + kTsDCol + h * NT + c * 16, v);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = tile_m * NT + c * 16 + j;
            if (row < args.M)
              dst[(int64_t)row * args.ldo] = __float2half_rn(
                  silu_mul_rounded(__uint_as_float(v[j]), xch[(c * 16 + j) * 128 + cl]));
          }
        }
      }
    } else if (ok && !*abort_flag) {
      const int h = (warp - 2) >> 2;
      const int u = 4 * h + (lane >> 3);
      const int e = u < 4 ? 2 * u : 2 * (u - 4) + 1;
      const int col = tile_n * BN + 8 * (8 * q + (lane & 7)) + e;
      const float bias = (args.bias && col < args.N) ? __half2float(args.bias[col]) : 0.f;
#pragma unroll
      for (int c = 0; c < NT / 16; ++c) {
        uint32_t v[16];
        sm100::tmem_ld_32x32b_x16(tmem + ((uint32_t)(32 * q) << 16) + kTsDCol + h * NT + c * 16, v);
        sm100::tmem_ld_wait();
        if (col < args.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = tile_m * NT + c * 16 + j;
            if (row < args.M) {
              if (args.splits > 1)
                args.part[((size_t)blockIdx.z * args.M + row) * args.N + col] = __uint_as_float(v[j]);
              else
                args.out[(int64_t)row * args.ldo + col] = __float2half_rn(__uint_as_float(v[j]) + bias);
            }
          }
        }
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    if (*abort_flag) sm100::mbar_wait_bounded(bar_accf, 0, nullptr, 100000000ull);
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTsTmemCols);
  }
}

// ---------------------------------------------------------------------------------
// host: tensor maps through the driver entry point (no link-time libcuda dependency)
// ---------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// out[M, N] = fp16(sum over z of part[z] (+ bias)), four columns per thread, z in order.
__global__ void __launch_bounds__(256)
tc_splitk_reduce(const float* __restrict__ part, int splits, int M, int N,
                 __half* __restrict__ out, int64_t ldo, const __half* __restrict__ bias) {
  const int n4 = N / 4;
  const int64_t total = (int64_t)M * n4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / n4;
    const int c = (int)(i - row * n4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int z = 0; z < splits; ++z) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(part + ((size_t)z * M + row) * N + c));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (bias) {
      acc.x += __half2float(bias[c]); acc.y += __half2float(bias[c + 1]);
      acc.z += __half2float(bias[c + 2]); acc.w += __half2float(bias[c + 3]);
    }
    const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
    *reinterpret_cast<uint2*>(out + row * ldo + c) = make_uint2(h2_as_u32(lo), h2_as_u32(hi));
  }
}

}  // namespace

// Split-K factor of the tcgen05 kernel: 1 when its output tiles already fill half the
// SMs; otherwise as many CTAs per tile as the SMs allow, at most 16, each with at least
// 8 K steps (512 rows) so that its pipeline still fills.
int tc_splits(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int64_t bm = M > 128 ? 256 : 128;
  const int64_t tiles = ((M + bm - 1) / bm) * ((N + BN - 1) / BN);
  if (tiles <= 0 || 2 * tiles >= num_sms) return 1;
  int64_t s = num_sms / tiles;
  if (s > K / BK / 8) s = K / BK / 8;
  if (s > 16) s = 16;
  return s < 1 ? 1 : (int)s;
}

// Stream-K schedule of the tcgen05 kernel, for output tiles that fill between half and
// most of one wave (down at M = 2048: 8 x 14 = 112 tiles on 148 SMs).  One CTA per tile
// runs the first S K steps; the other num_sms - tiles CTAs share the tiles' last K/64 - S
// steps evenly.  Every share is at least one tail long, so a tile has at most three parts
// (kSkSlots), and reaches at most kMaxSeg tiles.  Costs in K steps, from per-CTA timelines
// on B200 (a K step of a 256 x 256 tile takes ~0.85 us): a share pays kSkSegCost for each
// further tile it reaches (its 256 KB fp32 slot written while the other SMs stream their
// inputs: ~6.5 us), and the tile's last part kSkFixCost to sum the other slots and write
// fp16 (~11 us); one CTA per tile pays kTileEpiCost for its fp16 tile.  S minimises the
// larger of the two kinds of CTA.  Returns the tiles and sets *split = S, or returns 0
// when that saves less than a tenth.
constexpr int64_t kSkSegCost = 8, kSkFixCost = 12, kTileEpiCost = 3;
int64_t tc_streamk_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* split) {
  const int64_t bm = M > 128 ? 256 : 128;
  const int64_t tiles = ((M + bm - 1) / bm) * ((N + BN - 1) / BN);
  const int64_t kt = K / BK;
  if (tiles <= 0 || 2 * tiles < num_sms || tiles >= num_sms || tiles > kMaxCounters) return 0;
  const int64_t g2 = num_sms - tiles;
  int64_t best = -1, best_s = 0;
  for (int64_t s = (kt + 1) / 2; s < kt; ++s) {
    const int64_t L = kt - s;
    const int64_t lo = tiles * L / g2, hi = (tiles * L + g2 - 1) / g2;   // share lengths
    if (lo < L) continue;                       // a tail would reach three sharers
    const int64_t segs = (hi + L - 2) / L + 1;  // tiles a share of hi steps can reach
    if (segs > kMaxSeg) continue;
    const int64_t cost = std::max(s, hi + kSkSegCost * (segs - 1)) + kSkFixCost;
    if (best < 0 || cost < best) {
      best = cost;
      best_s = s;
    }
  }
  if (best < 0 || 10 * best > 9 * (kt + kTileEpiCost)) return 0;
  if (split) *split = (int)best_s;
  return tiles;
}

size_t tc_workspace_bytes(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int s = tc_splits(M, N, K, num_sms);
  if (s > 1) return kCounterRegionBytes + (size_t)s * M * N * sizeof(float);
  const int64_t sk = tc_streamk_plan(M, N, K, num_sms, nullptr);
  if (sk > 0) {
    const int64_t bm = M > 128 ? 256 : 128;
    return kCounterRegionBytes + (size_t)sk * kSkSlots * bm * BN * sizeof(float);
  }
  return 0;
}

bool tc_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                  const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size) {
  if (M < 1 || N < 32 || K < BK) return false;
  if (N % 32 || group_size % BK || K % group_size) return false;
  if (ldx % 8 || ldx < K) return false;
  if (!al16(x) || !al16(qweight) || !al16(qzeros) || !al16(scales)) return false;
  if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return false;
  return get_encode() != nullptr;
}

cudaError_t launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int M, int N, int K, int group_size, int num_sms, int* dev_status,
                           cudaStream_t stream, const char** why, const void* bias,
                           void* workspace, size_t workspace_bytes, bool silu) {
  *why = nullptr;
  if (silu && (N % (2 * BN) || bias)) {
    *why = "SiLU-mul epilogue needs N % 512 == 0 and no bias";
    return cudaSuccess;
  }
  if (!tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size)) {
    *why = "shape or alignment not supported";
    return cudaSuccess;
  }
  if (ldo % 8 || !al16(out)) {
    *why = "out must be 16-byte aligned with ldo % 8 == 0";
    return cudaSuccess;
  }
  const int nacc = M > 128 ? 2 : 1;
  const int BM = 128 * nacc;
  CUtensorMap tmA, tmW, tmS, tmZ;
  const int G = K / group_size;
  bool ok = make_map_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, K, M, (uint64_t)ldx * 2, BK, BM,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N / 8, K, (uint64_t)N / 2,
                        (silu ? BN / 16 : BN / 8), BK, CU_TENSOR_MAP_SWIZZLE_NONE) &&
            make_map_2d(&tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales, N, G, (uint64_t)N * 2,
                        (silu ? BN / 2 : BN), 1, CU_TENSOR_MAP_SWIZZLE_NONE) &&
            make_map_2d(&tmZ, CU_TENSOR_MAP_DATA_TYPE_INT32, qzeros, N / 8, G, (uint64_t)N / 2,
                        (silu ? BN / 16 : BN / 8), 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaSuccess;
  }
  static PerDeviceOnce attr_once;
  const cudaError_t attr_err = attr_once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Geo<1>::SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)Geo<2>::SMEM_BYTES);
    return e;
  });
  if (attr_err != cudaSuccess) return attr_err;
  TcArgs a;
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.M = M; a.N = N; a.K = K; a.gs = group_size;
  a.status = dev_status;
  a.bias = static_cast<const __half*>(bias);
  // split-K or stream-K when the caller's workspace holds the partials (after the decode
  // kernels' counter region, which must stay zero); otherwise one CTA per tile
  a.splits = silu ? 1 : tc_splits(M, N, K, num_sms);
  a.silu = silu ? 1 : 0;
  a.part = nullptr;
  a.streamk = 0;
  a.tiles_n = (N + BN - 1) / BN;
  a.sk_tiles = 0;
  a.sk_split = 0;
  a.persistent = 0;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_total = a.tiles_m * a.tiles_n;
  a.sk_part = nullptr;
  a.sk_cnt = nullptr;
  const bool ws_ok = workspace && al16(workspace) &&
                     workspace_bytes >= tc_workspace_bytes(M, N, K, num_sms);
  if (a.splits > 1) {
    if (ws_ok)
      a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegionBytes);
    else
      a.splits = 1;
  }
  dim3 grid((M + BM - 1) / BM, (N + BN - 1) / BN, a.splits);
  int sk_split = 0;
  const int64_t sk_tiles = a.splits == 1 && !silu ? tc_streamk_plan(M, N, K, num_sms, &sk_split) : 0;
  if (sk_tiles > 0 && ws_ok) {
    a.streamk = 1;
    a.sk_tiles = (int)sk_tiles;
    a.sk_split = sk_split;
    a.sk_cnt = static_cast<int*>(workspace);
    a.sk_part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegionBytes);
    grid = dim3(num_sms, 1, 1);
  } else if (a.splits == 1 && a.tiles_total > num_sms) {
    a.persistent = 1;                    // one CTA per SM, tiles taken in grid order
    grid = dim3(num_sms, 1, 1);
  }
  if (nacc == 2)
    gemm_tc_kernel<2><<<grid, kThreads, Geo<2>::SMEM_BYTES, stream>>>(tmA, tmW, tmS, tmZ, a);
  else
    gemm_tc_kernel<1><<<grid, kThreads, Geo<1>::SMEM_BYTES, stream>>>(tmA, tmW, tmS, tmZ, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.splits == 1) return e;
  tc_splitk_reduce<<<num_sms * 4, 256, 0, stream>>>(a.part, a.splits, M, N, a.out, ldo, a.bias);
  return cudaGetLastError();
}

// ---- small-M kernel ---------------------------------------------------------------------
int ts_tokens(int64_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : 64; }

// Split-K factor of the small-M kernel: as for the prefill kernel, but a CTA keeps at
// least 4 K steps (its ring is deeper than that, so every copy is issued at once), and
// tiles filling exactly half the SMs split in two (the gate+up shard of a 2-way tensor
// parallel MLP, 74 tiles: at M = 16 40.9 us unsplit, 29.7 us split).
int ts_splits(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int64_t nt = ts_tokens(M);
  const int64_t tiles = ((M + nt - 1) / nt) * ((N + BN - 1) / BN);
  if (tiles <= 0 || 2 * tiles > num_sms) return 1;
  int64_t s = num_sms / tiles;
  if (s > K / BK / kTsMinSteps) s = K / BK / kTsMinSteps;
  if (s > 16) s = 16;
  return s < 1 ? 1 : (int)s;
}

size_t ts_workspace_bytes(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int s = ts_splits(M, N, K, num_sms);
  return s > 1 ? kCounterRegionBytes + (size_t)s * M * N * sizeof(float) : 0;
}

bool ts_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                  const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size) {
  return M <= 64 && tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size);
}

cudaError_t launch_gemm_ts(const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int M, int N, int K, int group_size, int num_sms, int* dev_status,
                           cudaStream_t stream, const char** why, const void* bias,
                           void* workspace, size_t workspace_bytes, bool silu) {
  *why = nullptr;
  if (!ts_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size)) {
    *why = "shape or alignment not supported";
    return cudaSuccess;
  }
  if (silu && (N % (2 * BN) || bias || ts_splits(M, N, K, num_sms) != 1)) {
    *why = "SiLU-mul epilogue needs N a multiple of 512, no bias and no K split";
    return cudaSuccess;
  }
  if (ldo < (silu ? N / 2 : N)) {
    *why = silu ? "ldo must be at least N / 2" : "ldo must be at least N";
    return cudaSuccess;
  }
  const int nt = ts_tokens(M);
  CUtensorMap tmX, tmW, tmS, tmZ;
  const int G = K / group_size;
  bool ok = make_map_2d(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, K, M, (uint64_t)ldx * 2, BK, nt,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N / 8, K, (uint64_t)N / 2,
                        silu ? BN / 16 : BN / 8, BK,
                        silu ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales, N, G, (uint64_t)N * 2,
                        silu ? BN / 2 : BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE) &&
            make_map_2d(&tmZ, CU_TENSOR_MAP_DATA_TYPE_INT32, qzeros, N / 8, G, (uint64_t)N / 2,
                        silu ? BN / 16 : BN / 8, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaSuccess;
  }
  static PerDeviceOnce attr_once;
  const cudaError_t attr_err = attr_once.run([] {
    cudaError_t e = cudaFuncSetAttribute(gemm_ts_kernel<16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)TsGeo<16>::SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_ts_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TsGeo<32>::SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_ts_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TsGeo<64>::SMEM_BYTES);
    return e;
  });
  if (attr_err != cudaSuccess) return attr_err;
  TcArgs a;
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.M = M; a.N = N; a.K = K; a.gs = group_size;
  a.status = dev_status;
  a.bias = static_cast<const __half*>(bias);
  a.splits = ts_splits(M, N, K, num_sms);
  a.part = nullptr;
  a.silu = silu ? 1 : 0;
  if (a.splits > 1) {
    if (workspace && al16(workspace) && workspace_bytes >= ts_workspace_bytes(M, N, K, num_sms))
      a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegionBytes);
    else
      a.splits = 1;
  }
  dim3 grid((M + nt - 1) / nt, (N + BN - 1) / BN, a.splits);
  if (nt == 16)
    gemm_ts_kernel<16><<<grid, kThreads, TsGeo<16>::SMEM_BYTES, stream>>>(tmX, tmW, tmS, tmZ, a);
  else if (nt == 32)
    gemm_ts_kernel<32><<<grid, kThreads, TsGeo<32>::SMEM_BYTES, stream>>>(tmX, tmW, tmS, tmZ, a);
  else
    gemm_ts_kernel<64><<<grid, kThreads, TsGeo<64>::SMEM_BYTES, stream>>>(tmX, tmW, tmS, tmZ, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.splits == 1) return e;
  tc_splitk_reduce<<<num_sms * 4, 256, 0, stream>>>(a.part, a.splits, M, N, a.out, ldo, a.bias);
  return cudaGetLastError();
}

}  // namespace awq
