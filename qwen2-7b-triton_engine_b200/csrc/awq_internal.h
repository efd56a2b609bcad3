// awq_internal.h -- launch interfaces shared between the kernel files and the C-ABI
// layer (awq_capi.cu).  Not part of the public header.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace awq {

// Kernel attributes set with cudaFuncSetAttribute (the dynamic shared-memory limit) belong
// to the current device, so a process that drives several GPUs must set them on each:
// `run(set)` calls `set` once per device for this call site and returns its result on
// every later call on that device.
struct PerDeviceOnce {
  static constexpr int kDevices = 64;
  std::atomic<uint64_t> done{0};
  std::mutex mu;
  cudaError_t err[kDevices] = {};
  template <class F>
  cudaError_t run(F&& set) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kDevices) return cudaErrorInvalidDevice;
    if ((done.load(std::memory_order_acquire) >> dev) & 1u) return err[dev];
    std::lock_guard<std::mutex> lk(mu);
    if (!((done.load(std::memory_order_relaxed) >> dev) & 1u)) {
      err[dev] = set();
      done.fetch_or(uint64_t(1) << dev, std::memory_order_release);
    }
    return err[dev];
  }
};

// ---- dequant (awq_dequant.cu) -------------------------------------------------------
cudaError_t launch_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales,
                           void* out, int64_t K, int64_t N, int64_t group_size, int num_sms,
                           cudaStream_t stream);

// Split-K arrival counters sit at the head of the caller's workspace (the generic and
// the TMA decode kernels share the region); every kernel leaves the counters it used at
// zero.  One launch uses at most kMaxCounters of them.
constexpr int kMaxCounters = 16384;
constexpr size_t kCounterRegionBytes = kMaxCounters * sizeof(int);

// ---- decode / skinny GEMM on mma.sync (awq_gemv.cu) ----------------------------------
struct GemvPlan {
  int strips;      // ceil(N / 256): one warp-wide strip of 32 packed words each
  int splits;      // CTAs along K per strip (split-K)
  int bps;         // 8-row blocks of K per split
  int zchunks;     // token chunks of 16 (gridDim.z)
  int toksets;     // 4-token sets per chunk handled by one CTA (1, 2 or 4)
  int vec;         // 1: 16-byte loads of 4 packed words (N % 32 == 0, aligned)
  size_t smem;     // dynamic shared memory per CTA
  size_t ws_partials_bytes;  // fp32 split-K partials
  size_t ws_counter_bytes;   // int32 arrival counters (must start at zero)
};

// Returns false when the shape cannot be planned (the caller reports the error).
bool plan_gemv(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms, bool vec_ok,
               GemvPlan* plan);
size_t gemv_workspace_bytes(const GemvPlan& plan);
// plan_gemv with the split-K factor reduced until the workspace fits `max_workspace`
// bytes; false if even the smallest plan does not fit.
bool plan_gemv_bounded(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                       bool vec_ok, size_t max_workspace, GemvPlan* plan);
// `bias` (fp16 [N] or null) is added to every output row in fp32 before the fp16 rounding,
// here and in the other product kernels.
cudaError_t launch_gemv(const GemvPlan& plan, const void* x, int64_t ldx, const int32_t* qweight,
                        const int32_t* qzeros, const void* scales, void* out, int64_t ldo, int M,
                        int N, int K, int group_size, void* workspace, cudaStream_t stream,
                        const void* bias = nullptr);

// ---- decode on mma.sync with TMA streaming, one CTA per SM (awq_gemv_tma.cu) ---------
// Shapes TMA can describe (N % 32 == 0, 16-byte aligned qweight and x, ldx % 8 == 0).
bool gemv_tma_supported(const int32_t* qweight, int64_t N, int64_t ldx, const void* x);
struct GemvTmaPlan {
  int toksets;     // 4-token sets per CTA: 1 (M <= 4) or 2
  int strips;      // 256-column strips
  int tiles;       // strips x token chunks
  int grid;        // CTAs
  int base, extra; // CTAs per tile: the first `extra` tiles get base + 1, the rest base
  int xr;          // token rows reserved in shared memory
  int xs_stride;   // halves per staged token row
  int ngrp;        // zero / scale rows reserved in shared memory
  size_t smem;     // dynamic shared memory per CTA
  size_t ws_bytes; // workspace (counter region + fp32 split-K slots); 0 when no tile splits
};
// Plan of one launch of at most 16 tokens; false when the shape cannot be planned.
bool plan_gemv_tma(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                   GemvTmaPlan* plan);

// All-reduce across the ranks of a tensor-parallel group, fused into the decode kernel's
// epilogue (awq_tp.cu owns the buffers).  Rank r's receive buffer holds
//   state  int [2]                                     calls so far, tiles done this call
//   data   {fp32 value, u32 flag} [2][world][max_tiles][kArTileFloats]
// In call number e the last CTA of tile t stores every value of its fp32 tile, paired with
// the flag e + 1, as one 8-byte store into data[e % 2][rank][t] of every rank (peers over
// NVLink); each thread then polls, in its own buffer, the pairs of its elements from every
// rank until their flags read e + 1 and sums the values in rank order.  Flags are unique
// per call, so nothing is reset; two parities let a rank run one call ahead of a peer.
constexpr int kMaxWorld = 8;
constexpr int kArTileFloats = 8 * 256;    // tokens per tile x columns per tile
struct ArArgs {
  int world;                   // 1: no all-reduce
  int rank;
  int max_tiles;
  unsigned long long* data[kMaxWorld];   // rank r's data region (this rank's own included)
  int* state;                  // this rank's state words
  unsigned long long timeout_ns;
};
// silu_mul: out is [M, N/2] = silu(columns [0, N/2)) * columns [N/2, N) of the product,
// computed in the kernel's epilogue (needs gemv_tma_silu_ok and gemv_tma_silu_ws_bytes of
// workspace, zero-initialised counters included).
cudaError_t launch_gemv_tma(const GemvTmaPlan& plan, const void* x, int64_t ldx,
                            const int32_t* qweight, const int32_t* qzeros, const void* scales,
                            void* out, int64_t ldo, int M, int N, int K, int group_size,
                            void* workspace, int* dev_status, cudaStream_t stream,
                            const ArArgs* ar = nullptr, const void* bias = nullptr,
                            bool silu_mul = false);
bool gemv_tma_silu_ok(const GemvTmaPlan& plan, int64_t N);
size_t gemv_tma_silu_ws_bytes(const GemvTmaPlan& plan);

// ---- SiLU-mul of a [M, 2I] fp16 product (awq_silu.cu) ---------------------------------
// out[m, n] = fp16(silu(gu[m, n]) * gu[m, I + n]), fp32 math (the reference's
// kernels/silu_mul.py:41-64 on the two halves of model/qwen2.py:183-188).
cudaError_t launch_silu_mul(const void* gu, int64_t ldg, int M, int I, void* out, int64_t ldo,
                            int num_sms, cudaStream_t stream);
constexpr size_t kGemvTmaMaxSmem = 227 * 1024;   // sm_100's opt-in per-block maximum

// ---- prefill GEMM on tcgen05 / TMEM (awq_gemm_tc.cu) ----------------------------------
// Returns true when the tcgen05 kernel can run this shape (alignment / TMA rules).
bool tc_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                  const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size);
cudaError_t launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int M, int N, int K, int group_size, int num_sms, int* dev_status,
                           cudaStream_t stream, const char** why, const void* bias = nullptr,
                           void* workspace = nullptr, size_t workspace_bytes = 0,
                           bool silu = false);
// Split-K factor of the tcgen05 kernel and the workspace its fp32 partials need (0: none).
// With less workspace than this the kernel runs one CTA per output tile.
int tc_splits(int64_t M, int64_t N, int64_t K, int num_sms);
// Stream-K plan of the tcgen05 kernel: the tiles (0: not used) and, in *split, the K steps
// each tile CTA runs before the other CTAs share the tails.
int64_t tc_streamk_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* split);
size_t tc_workspace_bytes(int64_t M, int64_t N, int64_t K, int num_sms);

// ---- small-M GEMM on tcgen05 with the dequantized weights in TMEM (awq_gemm_tc.cu) ----
// M <= 64; same shape rules as the prefill kernel.  Tokens per CTA: 16, 32 or 64.
// silu: gate+up product with the SiLU-mul epilogue (out [M, N/2]; N a multiple of 512,
// no bias, only where the kernel runs without a K split).
bool ts_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                  const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size);
cudaError_t launch_gemm_ts(const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int M, int N, int K, int group_size, int num_sms, int* dev_status,
                           cudaStream_t stream, const char** why, const void* bias = nullptr,
                           void* workspace = nullptr, size_t workspace_bytes = 0,
                           bool silu = false);
int ts_tokens(int64_t M);
int ts_splits(int64_t M, int64_t N, int64_t K, int num_sms);
size_t ts_workspace_bytes(int64_t M, int64_t N, int64_t K, int num_sms);

// Receive-buffer layout of a tensor-parallel communicator (see ArArgs).
inline size_t tp_data_offset() { return 256; }
inline size_t tp_buffer_bytes(int world, int max_tiles) {
  return tp_data_offset() + (size_t)2 * world * max_tiles * kArTileFloats * 8;
}

// All-reduce of prefill-sized outputs (M > 16; communicators made with max_rows > 0).
// After the decode region come two fp16 planes of [max_rows][max_n]: `in`, where this
// rank's product kernel writes its partial output, and `res`, where the owner of each
// row slice (rank r owns rows [M r / world, M (r + 1) / world)) writes the summed rows.
// In the header: state words at kBigStateOffset ([0] calls so far, [1] CTAs past their
// slice this call, [2] CTAs done this call) and flags at kBigFlagOffset (in_flag[world]
// then res_flag[world], written by the other ranks: the call number + 1 of the latest
// call whose input / summed slice that rank has published).
constexpr size_t kBigStateOffset = 64, kBigFlagOffset = 128;
inline size_t tp_big_offset(int world, int max_tiles) {
  return (tp_buffer_bytes(world, max_tiles) + 255) / 256 * 256;
}
inline size_t tp_big_plane_bytes(int64_t max_rows, int64_t max_n) {
  return ((size_t)max_rows * max_n * 2 + 255) / 256 * 256;
}

}  // namespace awq
struct awq_tp_comm;
namespace awq {
// Kernel arguments of a ready communicator (false when it is not opened).
bool tp_ar_args(const awq_tp_comm* comm, ArArgs* args);
// This rank's `in` plane (null when the communicator has no prefill region), and the
// all-reduce of the fp16 [M, N] partials the ranks wrote there into out (row stride
// ldo): reduce-scatter by row slices, all-gather through the `res` planes.
void* tp_big_in_plane(const awq_tp_comm* comm);
cudaError_t launch_tp_big_allreduce(const awq_tp_comm* comm, int M, int N, void* out, int64_t ldo,
                                    int num_sms, int* dev_status, cudaStream_t stream);

// Sets the message awq_last_error() returns on this thread; returns `code`.
int set_last_error(int code, const char* msg);

}  // namespace awq

// Tensor-parallel communicator behind the C ABI's opaque awq_tp_comm (awq_tp.cu).
struct awq_tp_comm {
  int device = 0, world = 1, rank = 0;
  int64_t max_n = 0;
  int64_t max_rows = 0;                    // rows of the prefill all-reduce planes (0: none)
  int max_tiles = 0;
  size_t bytes = 0;
  void* local = nullptr;                   // this rank's receive buffer
  void* peer[awq::kMaxWorld] = {};         // every rank's buffer as mapped here
  bool opened[awq::kMaxWorld] = {};        // peer[r] came from cudaIpcOpenMemHandle
  unsigned long long timeout_ns = 2000000000ull;
  bool ready = false;                      // awq_tp_comm_open succeeded
};
