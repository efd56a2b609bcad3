// awq_internal.h -- launch interfaces shared between the kernel files and the C-ABI
// layer (awq_capi.cu).  Not part of the public header.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace awq {

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
cudaError_t launch_gemv(const GemvPlan& plan, const void* x, int64_t ldx, const int32_t* qweight,
                        const int32_t* qzeros, const void* scales, void* out, int64_t ldo, int M,
                        int N, int K, int group_size, void* workspace, cudaStream_t stream);

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
cudaError_t launch_gemv_tma(const GemvTmaPlan& plan, const void* x, int64_t ldx,
                            const int32_t* qweight, const int32_t* qzeros, const void* scales,
                            void* out, int64_t ldo, int M, int N, int K, int group_size,
                            void* workspace, int* dev_status, cudaStream_t stream);
constexpr size_t kGemvTmaMaxSmem = 227 * 1024;   // sm_100's opt-in per-block maximum

// ---- prefill GEMM on tcgen05 / TMEM (awq_gemm_tc.cu) ----------------------------------
// Returns true when the tcgen05 kernel can run this shape (alignment / TMA rules).
bool tc_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                  const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size);
cudaError_t launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int M, int N, int K, int group_size, int num_sms, int* dev_status,
                           cudaStream_t stream, const char** why);

// Sets the message awq_last_error() returns on this thread; returns `code`.
int set_last_error(int code, const char* msg);

}  // namespace awq
