// awq_capi.cu -- extern "C" entry points of libawq_b200.so (declared in include/awq_b200.h).
//
// Validation, kernel choice and workspace accounting for the AWQ W4A16 product.  The
// Python drop-in (kernels/awq_gemm.py in this package) calls these through ctypes; a
// C/C++ host can link them directly.  Mirrors the dispatch of awq_gemm_forward
// (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:237-284) with the decode /
// prefill split moved from M <= 4 to M <= 16 and both branches replaced by sm_100a
// kernels that read the packed weights directly.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/awq_b200.h"
#include "awq_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  return fail(AWQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

__device__ int g_device_status;   // one per device; kernels OR their error bits in

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int num_sms = 0;
  int* status = nullptr;
  bool ready = false;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(AWQ_ERR_UNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int sms = 0, major = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail_cuda(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return fail_cuda(e, "cudaDeviceGetAttribute");
    if (major != 10)
      return fail(AWQ_ERR_UNSUPPORTED, "device %d has compute capability %d.x; this library is built for sm_100a",
                  dev, major);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(status)");
    d.num_sms = sms;
    d.status = static_cast<int*>(p);
    d.ready = true;
  }
  *out = &d;
  return AWQ_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_weights(const int32_t* qweight, const int32_t* qzeros, const void* scales, int64_t K,
                  int64_t N, int64_t group_size) {
  if (!qweight || !qzeros || !scales) return fail(AWQ_ERR_INVALID_ARG, "null weight pointer");
  if (K <= 0 || N <= 0) return fail(AWQ_ERR_INVALID_ARG, "K=%lld N=%lld must be positive", (long long)K, (long long)N);
  if (N % 8) return fail(AWQ_ERR_INVALID_ARG, "N=%lld is not a multiple of 8", (long long)N);
  if (group_size <= 0 || group_size % 8)
    return fail(AWQ_ERR_INVALID_ARG, "group_size=%lld must be a positive multiple of 8", (long long)group_size);
  if (K % group_size)
    return fail(AWQ_ERR_INVALID_ARG, "K=%lld is not a multiple of group_size=%lld", (long long)K, (long long)group_size);
  if (K > (int64_t)1 << 30 || N > (int64_t)1 << 30)
    return fail(AWQ_ERR_INVALID_ARG, "K or N above 2^30");
  if (!aligned16(qweight) || !aligned16(qzeros) || !aligned16(scales))
    return fail(AWQ_ERR_INVALID_ARG, "qweight, qzeros and scales must be 16-byte aligned");
  return AWQ_OK;
}

}  // namespace

int awq::set_last_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

extern "C" {

int awq_version(void) { return 100; }

const char* awq_last_error(void) { return g_last_error.c_str(); }

int awq_dequant_f16(const int32_t* qweight, const int32_t* qzeros, const void* scales, void* out,
                    int64_t K, int64_t N, int64_t group_size, void* stream) {
  int rc = check_weights(qweight, qzeros, scales, K, N, group_size);
  if (rc) return rc;
  if (!out || !aligned16(out)) return fail(AWQ_ERR_INVALID_ARG, "out must be a 16-byte aligned pointer");
  DeviceInfo* d = nullptr;
  if ((rc = device_info(&d))) return rc;
  cudaError_t e = awq::launch_dequant(qweight, qzeros, scales, out, K, N, group_size, d->num_sms,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, "dequant launch");
  return AWQ_OK;
}

size_t awq_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size) {
  DeviceInfo* d = nullptr;
  if (device_info(&d)) return 0;
  size_t need = 0;
  awq::GemvPlan plan;
  // generic decode kernel (the unaligned, scalar-load plan has the same grid)
  if (awq::plan_gemv(M, N, K, group_size, d->num_sms, true, &plan))
    need = awq::gemv_workspace_bytes(plan);
  // TMA decode kernel: launches of 16 tokens and one of the remainder
  for (const int64_t mc : {M < 16 ? M : (int64_t)16, M > 16 ? M % 16 : (int64_t)0}) {
    awq::GemvTmaPlan tp;
    if (mc > 0 && awq::plan_gemv_tma(mc, N, K, group_size, d->num_sms, &tp) && tp.ws_bytes > need)
      need = tp.ws_bytes;
  }
  // tcgen05 kernels' split-K partials
  if (M > 16) {
    const size_t tc = awq::tc_workspace_bytes(M, N, K, d->num_sms);
    if (tc > need) need = tc;
  }
  if (M <= 64) {
    const size_t ts = awq::ts_workspace_bytes(M, N, K, d->num_sms);
    if (ts > need) need = ts;
  }
  return need;
}

int awq_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  if (workspace_bytes == 0) return AWQ_OK;
  if (!workspace) return fail(AWQ_ERR_INVALID_ARG, "null workspace");
  cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(workspace)");
  return AWQ_OK;
}

int awq_tc_schedule(int64_t M, int64_t N, int64_t K, int num_sms, int* kind, int* param) {
  if (!kind || !param) return fail(AWQ_ERR_INVALID_ARG, "null kind or param");
  if (M <= 0 || N <= 0 || K < 64 || K % 64 || num_sms <= 0 || M > (int64_t)1 << 30 ||
      N > (int64_t)1 << 30 || K > (int64_t)1 << 30)
    return fail(AWQ_ERR_INVALID_ARG, "M=%lld N=%lld K=%lld num_sms=%d out of range", (long long)M,
                (long long)N, (long long)K, num_sms);
  const int s = awq::tc_splits(M, N, K, num_sms);
  if (s > 1) {
    *kind = AWQ_TC_SPLITK;
    *param = s;
    return AWQ_OK;
  }
  int split = 0;
  if (awq::tc_streamk_plan(M, N, K, num_sms, &split) > 0) {
    *kind = AWQ_TC_STREAMK;
    *param = split;
    return AWQ_OK;
  }
  const int64_t bm = M > 128 ? 256 : 128;
  const int64_t tiles = ((M + bm - 1) / bm) * ((N + 255) / 256);
  *kind = tiles > num_sms ? AWQ_TC_PERSISTENT : AWQ_TC_GRID;
  *param = (int)tiles;
  return AWQ_OK;
}

int awq_tc_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                     const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size) {
  return awq::tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size) ? 1 : 0;
}

// The product behind awq_gemm_f16_ex and awq_gemm_f16_bias (bias: fp16 [N] or null).
static int gemm_impl(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                     const void* scales, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                     int64_t group_size, void* workspace, size_t workspace_bytes, void* stream,
                     int path, const void* bias) {
  int rc = check_weights(qweight, qzeros, scales, K, N, group_size);
  if (rc) return rc;
  if (!x || !out) return fail(AWQ_ERR_INVALID_ARG, "null x or out");
  if (M <= 0 || M > (int64_t)1 << 30) return fail(AWQ_ERR_INVALID_ARG, "M=%lld out of range", (long long)M);
  if (ldx < K || ldo < N) return fail(AWQ_ERR_INVALID_ARG, "ldx < K or ldo < N");
  if ((reinterpret_cast<uintptr_t>(x) & 1) || (reinterpret_cast<uintptr_t>(out) & 1))
    return fail(AWQ_ERR_INVALID_ARG, "x and out must be 2-byte aligned");
  if (path != AWQ_PATH_AUTO && path != AWQ_PATH_DECODE && path != AWQ_PATH_TC &&
      path != AWQ_PATH_TS)
    return fail(AWQ_ERR_INVALID_ARG, "unknown path %d", path);
  DeviceInfo* d = nullptr;
  if ((rc = device_info(&d))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Small-M tcgen05 kernel (weights dequantized into TMEM): measured on B200 it beats the
  // decode kernel from 9 to 16 tokens on every Qwen2-7B shape (M = 9: o 11.0 vs 14.8 us,
  // gate+up 37.0 vs 48.0, down 24.9 vs 31.5; the decode kernel reads the weights once per
  // 8 tokens) and the prefill kernel on gate+up (37 vs 47 us).  Above 16 tokens it is
  // within 5 % of the split prefill kernel, which keeps that range.
  if (path == AWQ_PATH_AUTO && M > 8 && M <= 16 &&
      awq::ts_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size)) {
    const int s = awq::ts_splits(M, N, K, d->num_sms);
    const bool ws_ok = s == 1 || (workspace && aligned16(workspace) &&
                                  workspace_bytes >= awq::ts_workspace_bytes(M, N, K, d->num_sms));
    if (ws_ok) path = AWQ_PATH_TS;
  }
  if (path == AWQ_PATH_TS) {
    if (!awq::ts_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size))
      return fail(AWQ_ERR_UNSUPPORTED, "small-M tcgen05 path cannot run M=%lld N=%lld K=%lld gs=%lld with these pointers",
                  (long long)M, (long long)N, (long long)K, (long long)group_size);
    const char* why = nullptr;
    cudaError_t e = awq::launch_gemm_ts(x, ldx, qweight, qzeros, scales, out, ldo, (int)M, (int)N,
                                        (int)K, (int)group_size, d->num_sms, d->status, st, &why,
                                        bias, workspace, workspace_bytes);
    if (why) return fail(AWQ_ERR_UNSUPPORTED, "small-M tcgen05 path: %s", why);
    if (e != cudaSuccess) return fail_cuda(e, "small-M tcgen05 GEMM launch");
    return AWQ_OK;
  }

  bool use_tc = false;
  if (path == AWQ_PATH_TC) {
    if (!awq::tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size))
      return fail(AWQ_ERR_UNSUPPORTED, "tcgen05 path cannot run M=%lld N=%lld K=%lld gs=%lld with these pointers",
                  (long long)M, (long long)N, (long long)K, (long long)group_size);
    use_tc = true;
  } else if (path == AWQ_PATH_AUTO) {
    // The tcgen05 kernel runs ceil(M / BM) x ceil(N / 256) output tiles (BM 128, or 256
    // above M = 128), split along K when they cannot fill the GPU and the workspace holds
    // the partials.  Without the split, few tiles (o, q/k/v, down at small M) lose to the
    // decode kernel in 16-token launches up to M = 64 (measured on B200: down at M = 24 /
    // 32 takes 55 / 63 us there against 173 us with 14 unsplit tcgen05 CTAs, 26 / 27 us
    // split ten ways).
    const int64_t bm = M > 128 ? 256 : 128;
    int64_t tc_ctas = ((M + bm - 1) / bm) * ((N + 255) / 256);
    const size_t tc_need = awq::tc_workspace_bytes(M, N, K, d->num_sms);
    if (tc_need > 0 && workspace && workspace_bytes >= tc_need)
      tc_ctas *= awq::tc_splits(M, N, K, d->num_sms);
    use_tc = M > 16 && (M > 64 || 2 * tc_ctas >= d->num_sms) &&
             awq::tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size);
  }

  if (use_tc) {
    const char* why = nullptr;
    cudaError_t e = awq::launch_gemm_tc(x, ldx, qweight, qzeros, scales, out, ldo, (int)M, (int)N,
                                        (int)K, (int)group_size, d->num_sms, d->status, st, &why,
                                        bias, workspace, workspace_bytes);
    if (why) return fail(AWQ_ERR_UNSUPPORTED, "tcgen05 path: %s", why);
    if (e != cudaSuccess) return fail_cuda(e, "tcgen05 GEMM launch");
    return AWQ_OK;
  }

  if (awq::gemv_tma_supported(qweight, N, ldx, x)) {
    // launches of at most 16 tokens (one plan for full chunks, one for the remainder)
    awq::GemvTmaPlan full = {}, rest = {};
    const int64_t m_full = M < 16 ? M : 16, m_rest = M > 16 ? M % 16 : 0;
    const bool planned = awq::plan_gemv_tma(m_full, N, K, group_size, d->num_sms, &full) &&
                         (m_rest == 0 || awq::plan_gemv_tma(m_rest, N, K, group_size, d->num_sms, &rest));
    if (planned) {
      size_t need = full.ws_bytes;
      if (m_rest > 0 && rest.ws_bytes > need) need = rest.ws_bytes;
      if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(AWQ_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
      if (need > 0 && !aligned16(workspace))
        return fail(AWQ_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
      const char* xb = static_cast<const char*>(x);            // fp16 rows: 2 bytes each
      char* ob = static_cast<char*>(out);
      for (int64_t m0 = 0; m0 < M; m0 += 16) {
        const int64_t mc = M - m0 < 16 ? M - m0 : 16;
        cudaError_t e = awq::launch_gemv_tma(mc == m_full ? full : rest, xb + 2 * m0 * ldx, ldx,
                                             qweight, qzeros, scales, ob + 2 * m0 * ldo, ldo, (int)mc,
                                             (int)N, (int)K, (int)group_size, workspace, d->status,
                                             st, nullptr, bias);
        if (e != cudaSuccess) return fail_cuda(e, "decode (TMA) kernel launch");
      }
      return AWQ_OK;
    }
  }

  const bool vec_ok = (N % 32 == 0) && aligned16(qweight);
  awq::GemvPlan plan;
  if (!awq::plan_gemv(M, N, K, group_size, d->num_sms, vec_ok, &plan))
    return fail(AWQ_ERR_UNSUPPORTED, "no decode plan for M=%lld N=%lld K=%lld", (long long)M,
                (long long)N, (long long)K);
  const size_t need = awq::gemv_workspace_bytes(plan);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(AWQ_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (need > 0 && !aligned16(workspace))
    return fail(AWQ_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  cudaError_t e = awq::launch_gemv(plan, x, ldx, qweight, qzeros, scales, out, ldo, (int)M, (int)N,
                                   (int)K, (int)group_size, workspace, st, bias);
  if (e != cudaSuccess) return fail_cuda(e, "decode kernel launch");
  return AWQ_OK;
}

int awq_gemm_f16_ex(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                    const void* scales, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                    int64_t group_size, void* workspace, size_t workspace_bytes, void* stream,
                    int path) {
  return gemm_impl(x, ldx, qweight, qzeros, scales, out, ldo, M, N, K, group_size, workspace,
                   workspace_bytes, stream, path, nullptr);
}

int awq_gemm_f16_bias(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                      const void* scales, const void* bias, void* out, int64_t ldo, int64_t M,
                      int64_t N, int64_t K, int64_t group_size, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!bias || (reinterpret_cast<uintptr_t>(bias) & 1))
    return fail(AWQ_ERR_INVALID_ARG, "bias must be a non-null, 2-byte aligned fp16 [N] pointer");
  return gemm_impl(x, ldx, qweight, qzeros, scales, out, ldo, M, N, K, group_size, workspace,
                   workspace_bytes, stream, AWQ_PATH_AUTO, bias);
}

// ---- gate+up product followed by SiLU-mul --------------------------------------------
// The fused decode plan (pair epilogue) when the shape allows it; the TMA kernel's pointer
// rules are checked separately, by the caller that has the pointers.
static bool silu_fused_plan(int64_t M, int64_t N, int64_t K, int64_t group_size, int num_sms,
                            awq::GemvTmaPlan* p) {
  return M >= 1 && M <= 8 && awq::plan_gemv_tma(M, N, K, group_size, num_sms, p) &&
         awq::gemv_tma_silu_ok(*p, N);
}

// Offset of the unfused path's fp16 [M, N] product inside the workspace: after the
// product's own workspace and never inside the counter region the other calls share.
static size_t silu_temp_offset(int64_t M, int64_t N, int64_t K, int64_t group_size) {
  size_t off = awq_gemm_workspace_bytes(M, N, K, group_size);
  off = (off + 255) / 256 * 256;
  return off < awq::kCounterRegionBytes ? awq::kCounterRegionBytes : off;
}

size_t awq_gemm_silu_mul_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size) {
  DeviceInfo* d = nullptr;
  if (device_info(&d) || M <= 0 || N <= 0 || K <= 0) return 0;
  size_t need = silu_temp_offset(M, N, K, group_size) + (size_t)M * N * 2;
  awq::GemvTmaPlan p;
  if (silu_fused_plan(M, N, K, group_size, d->num_sms, &p)) {
    const size_t fused = awq::gemv_tma_silu_ws_bytes(p);
    if (fused > need) need = fused;
  }
  return need;
}

int awq_gemm_f16_silu_mul(const void* x, int64_t ldx, const int32_t* qweight,
                          const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                          int64_t M, int64_t N, int64_t K, int64_t group_size, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_weights(qweight, qzeros, scales, K, N, group_size);
  if (rc) return rc;
  if (!x || !out) return fail(AWQ_ERR_INVALID_ARG, "null x or out");
  if (M <= 0 || M > (int64_t)1 << 30) return fail(AWQ_ERR_INVALID_ARG, "M=%lld out of range", (long long)M);
  if (N % 2) return fail(AWQ_ERR_INVALID_ARG, "N=%lld is not even (gate and up halves)", (long long)N);
  if (ldx < K || ldo < N / 2) return fail(AWQ_ERR_INVALID_ARG, "ldx < K or ldo < N/2");
  if ((reinterpret_cast<uintptr_t>(x) & 1) || (reinterpret_cast<uintptr_t>(out) & 1))
    return fail(AWQ_ERR_INVALID_ARG, "x and out must be 2-byte aligned");
  if (!workspace || !aligned16(workspace))
    return fail(AWQ_ERR_INVALID_ARG, "a 16-byte aligned workspace is required");
  DeviceInfo* d = nullptr;
  if ((rc = device_info(&d))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  awq::GemvTmaPlan p;
  if (awq::gemv_tma_supported(qweight, N, ldx, x) &&
      silu_fused_plan(M, N, K, group_size, d->num_sms, &p)) {
    const size_t need = awq::gemv_tma_silu_ws_bytes(p);
    if (workspace_bytes < need)
      return fail(AWQ_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    cudaError_t e = awq::launch_gemv_tma(p, x, ldx, qweight, qzeros, scales, out, ldo, (int)M,
                                         (int)N, (int)K, (int)group_size, workspace, d->status,
                                         st, nullptr, nullptr, /*silu_mul=*/true);
    if (e != cudaSuccess) return fail_cuda(e, "decode (TMA) kernel launch, SiLU-mul epilogue");
    return AWQ_OK;
  }
  // From 9 to 16 tokens the product runs on the small-M tcgen05 kernel; when it runs
  // without a K split (every Qwen2-7B gate+up call), its epilogue does the SiLU-mul the
  // same way: each CTA's 256 columns are 128 gate and the matching 128 up columns.
  if (M > 8 && M <= 16 && N % 512 == 0 &&
      awq::ts_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size) &&
      awq::ts_splits(M, N, K, d->num_sms) == 1) {
    const char* why = nullptr;
    cudaError_t e = awq::launch_gemm_ts(x, ldx, qweight, qzeros, scales, out, ldo, (int)M,
                                        (int)N, (int)K, (int)group_size, d->num_sms, d->status,
                                        st, &why, nullptr, nullptr, 0, /*silu=*/true);
    if (why) return fail(AWQ_ERR_UNSUPPORTED, "small-M tcgen05 SiLU-mul path: %s", why);
    if (e != cudaSuccess) return fail_cuda(e, "small-M tcgen05 GEMM launch, SiLU-mul epilogue");
    return AWQ_OK;
  }
  // Above 16 tokens, when the product would run on the tcgen05 kernel unsplit (its tiles
  // fill at least half the SMs: every Qwen2-7B gate+up call), that kernel's epilogue does
  // the SiLU-mul: a tile holds 128 gate and the matching 128 up columns, and only the
  // [M, N/2] result is written.
  if (M > 16 && N % 512 == 0 && aligned16(out) && ldo % 8 == 0 &&
      awq::tc_supported(x, ldx, qweight, qzeros, scales, M, N, K, group_size)) {
    const int64_t bm = M > 128 ? 256 : 128;
    const int64_t tiles = ((M + bm - 1) / bm) * (N / 256);
    if (2 * tiles >= d->num_sms) {
      const char* why = nullptr;
      cudaError_t e = awq::launch_gemm_tc(x, ldx, qweight, qzeros, scales, out, ldo, (int)M,
                                          (int)N, (int)K, (int)group_size, d->num_sms, d->status,
                                          st, &why, nullptr, nullptr, 0, /*silu=*/true);
      if (why) return fail(AWQ_ERR_UNSUPPORTED, "tcgen05 SiLU-mul path: %s", why);
      if (e != cudaSuccess) return fail_cuda(e, "tcgen05 GEMM launch, SiLU-mul epilogue");
      return AWQ_OK;
    }
  }
  const size_t off = silu_temp_offset(M, N, K, group_size);
  const size_t need = off + (size_t)M * N * 2;
  if (workspace_bytes < need)
    return fail(AWQ_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  void* prod = static_cast<char*>(workspace) + off;
  rc = gemm_impl(x, ldx, qweight, qzeros, scales, prod, N, M, N, K, group_size, workspace, off,
                 stream, AWQ_PATH_AUTO, nullptr);
  if (rc) return rc;
  cudaError_t e = awq::launch_silu_mul(prod, N, (int)M, (int)(N / 2), out, ldo, d->num_sms, st);
  if (e != cudaSuccess) return fail_cuda(e, "SiLU-mul kernel launch");
  return AWQ_OK;
}

int awq_gemm_f16(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                 const void* scales, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                 int64_t group_size, void* workspace, size_t workspace_bytes, void* stream) {
  return awq_gemm_f16_ex(x, ldx, qweight, qzeros, scales, out, ldo, M, N, K, group_size, workspace,
                         workspace_bytes, stream, AWQ_PATH_AUTO);
}

int awq_allreduce_supported(const awq_tp_comm* comm, const void* x, int64_t ldx,
                            const int32_t* qweight, int64_t M, int64_t N, int64_t K,
                            int64_t group_size) {
  DeviceInfo* d = nullptr;
  if (!comm || !comm->ready || device_info(&d)) return 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return 0;
  if (M <= 0 || N <= 0 || N > comm->max_n || group_size <= 0 || K <= 0 || K % group_size) return 0;
  if (M > 16) return M <= comm->max_rows && N <= comm->max_n && N % 8 == 0 ? 1 : 0;
  if (!awq::gemv_tma_supported(qweight, N, ldx, x)) return 0;
  // every launch must run its CTAs in one wave: a tile's last CTA waits for the other
  // ranks, and must never hold an SM that a not-yet-started CTA of its own grid needs
  for (const int64_t mc : {M < 16 ? M : (int64_t)16, M > 16 ? M % 16 : (int64_t)0}) {
    if (mc == 0) continue;
    awq::GemvTmaPlan p;
    if (!awq::plan_gemv_tma(mc, N, K, group_size, d->num_sms, &p) || p.grid > d->num_sms ||
        p.tiles > comm->max_tiles)
      return 0;
  }
  return 1;
}

int awq_gemm_f16_allreduce(awq_tp_comm* comm, const void* x, int64_t ldx, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                           int64_t M, int64_t N, int64_t K, int64_t group_size, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int rc = check_weights(qweight, qzeros, scales, K, N, group_size);
  if (rc) return rc;
  if (!comm || !comm->ready) return fail(AWQ_ERR_INVALID_ARG, "communicator missing or not opened");
  if (!x || !out) return fail(AWQ_ERR_INVALID_ARG, "null x or out");
  if (M <= 0 || M > (int64_t)1 << 30) return fail(AWQ_ERR_INVALID_ARG, "M=%lld out of range", (long long)M);
  if (ldx < K || ldo < N) return fail(AWQ_ERR_INVALID_ARG, "ldx < K or ldo < N");
  if ((reinterpret_cast<uintptr_t>(out) & 1)) return fail(AWQ_ERR_INVALID_ARG, "out must be 2-byte aligned");
  if (!awq_allreduce_supported(comm, x, ldx, qweight, M, N, K, group_size))
    return fail(AWQ_ERR_UNSUPPORTED, "fused all-reduce cannot run M=%lld N=%lld K=%lld gs=%lld here "
                "(see awq_allreduce_supported)", (long long)M, (long long)N, (long long)K,
                (long long)group_size);
  DeviceInfo* d = nullptr;
  if ((rc = device_info(&d))) return rc;
  if (M > 16) {
    // prefill-sized: the product into this rank's plane, then the all-reduce kernel
    if (!aligned16(out) || ldo % 8)
      return fail(AWQ_ERR_INVALID_ARG, "out must be 16-byte aligned with ldo %% 8 == 0 above 16 tokens");
    void* plane = awq::tp_big_in_plane(comm);
    rc = gemm_impl(x, ldx, qweight, qzeros, scales, plane, N, M, N, K, group_size, workspace,
                   workspace_bytes, stream, AWQ_PATH_AUTO, nullptr);
    if (rc) return rc;
    cudaError_t e = awq::launch_tp_big_allreduce(comm, (int)M, (int)N, out, ldo, d->num_sms,
                                                 d->status, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail_cuda(e, "all-reduce kernel launch");
    return AWQ_OK;
  }
  awq::ArArgs ar;
  if (!awq::tp_ar_args(comm, &ar)) return fail(AWQ_ERR_INVALID_ARG, "communicator not opened");
  awq::GemvTmaPlan full = {}, rest = {};
  const int64_t m_full = M < 16 ? M : 16, m_rest = M > 16 ? M % 16 : 0;
  awq::plan_gemv_tma(m_full, N, K, group_size, d->num_sms, &full);
  if (m_rest) awq::plan_gemv_tma(m_rest, N, K, group_size, d->num_sms, &rest);
  size_t need = full.ws_bytes;
  if (m_rest > 0 && rest.ws_bytes > need) need = rest.ws_bytes;
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(AWQ_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (need > 0 && !aligned16(workspace))
    return fail(AWQ_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* xb = static_cast<const char*>(x);
  char* ob = static_cast<char*>(out);
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int64_t mc = M - m0 < 16 ? M - m0 : 16;
    cudaError_t e = awq::launch_gemv_tma(mc == m_full ? full : rest, xb + 2 * m0 * ldx, ldx, qweight,
                                         qzeros, scales, ob + 2 * m0 * ldo, ldo, (int)mc, (int)N,
                                         (int)K, (int)group_size, workspace, d->status, st, &ar);
    if (e != cudaSuccess) return fail_cuda(e, "fused all-reduce kernel launch");
  }
  return AWQ_OK;
}

int awq_device_status(void* stream, int* status_out) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail_cuda(e, "reading device status");
  if (v) {
    const int zero = 0;
    e = cudaMemcpyAsync(d->status, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda(e, "clearing device status");
  }
  if (status_out) *status_out = v;
  if (v) return fail(AWQ_ERR_DEVICE, "kernel status word = %d", v);
  return AWQ_OK;
}

}  // extern "C"
