// awq_noalloc.cu -- an AWQ W4A16 entry point that allocates no device memory.
//
// Some callers cannot allocate device memory on the path where they run the product:
// an engine that pre-plans every byte of device memory and forbids libraries from
// allocating on its decode loop (cudaMalloc / cudaFree can synchronize the device and
// stall every stream), or a host framework whose plugin interface hands a library only
// input and output buffers and no allocator.  awq_gemm_f16_noalloc serves them: the
// caller passes x, the packed weights and out, and the split-K scratch of the generic
// decode kernel (partial sums and arrival counters) lives in a file-scope device array
// that every GPU loading this library holds until the process exits.
//
// Limits and rules (also stated in include/awq_b200.h):
//   * scratch = kNoAllocScratchBytes (4 MiB) per device; the split-K factor is reduced
//     until the partial sums fit, and a shape that does not fit even then is rejected
//     with AWQ_ERR_WORKSPACE and a message naming the size it would need;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) -- make that first call before
//     any stream capture;
//   * the split-K counters at the head of the array start at zero because a __device__
//     array is zero-initialised when the module loads, and the generic kernel (which has
//     no wait that can give up) leaves every counter it used at zero; nothing here writes
//     the array from the host;
//   * every call shares the one array; calls that overlap on the GPU (different streams,
//     or graph branches without an order between them) race on it and give wrong
//     results.
// The kernel is the generic decode kernel of awq_gemv.cu (mma.sync, split-K); any M is
// accepted (16-row chunks), so large M is correct but slow here.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/awq_b200.h"
#include "awq_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;              // 4 MiB per device

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
  void* ptr = nullptr;     // device address of g_noalloc_scratch on this device
  int num_sms = 0;
  bool ready = false;
};
constexpr int kMaxDevices = 64;
ScratchSlot g_slot[kMaxDevices];
std::mutex g_slot_mu;

int fail(int code, const char* msg) { return awq::set_last_error(code, msg); }

int slot_for_current_device(ScratchSlot** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(AWQ_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(AWQ_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_slot_mu);
  ScratchSlot& s = g_slot[dev];
  if (!s.ready) {
    // The symbol is a host-side stand-in; the kernel needs the device address, looked
    // up here with this device current.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail(AWQ_ERR_CUDA, cudaGetErrorString(e));
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(AWQ_ERR_CUDA, cudaGetErrorString(e));
    s.ptr = p;
    s.num_sms = sms;
    s.ready = true;
  }
  *out = &s;
  return AWQ_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int awq_gemm_f16_noalloc(const void* x, int64_t ldx, const int32_t* qweight,
                                    const int32_t* qzeros, const void* scales, void* out,
                                    int64_t ldo, int64_t M, int64_t N, int64_t K,
                                    int64_t group_size, void* stream) {
  if (!x || !qweight || !qzeros || !scales || !out) return fail(AWQ_ERR_INVALID_ARG, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || N % 8 || group_size <= 0 || group_size % 8 || K % group_size)
    return fail(AWQ_ERR_INVALID_ARG,
                "need M, N, K > 0, N % 8 == 0, group_size % 8 == 0 and K % group_size == 0");
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30 || K > (int64_t)1 << 30)
    return fail(AWQ_ERR_INVALID_ARG, "M, N or K above 2^30");
  if (ldx < K || ldo < N) return fail(AWQ_ERR_INVALID_ARG, "ldx < K or ldo < N");
  if (!al16(qweight) || !al16(qzeros) || !al16(scales))
    return fail(AWQ_ERR_INVALID_ARG, "qweight, qzeros and scales must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(x) & 1) || (reinterpret_cast<uintptr_t>(out) & 1))
    return fail(AWQ_ERR_INVALID_ARG, "x and out must be 2-byte aligned");

  ScratchSlot* slot = nullptr;
  int rc = slot_for_current_device(&slot);
  if (rc) return rc;

  const bool vec_ok = (N % 32 == 0) && al16(qweight);
  awq::GemvPlan plan;
  if (!awq::plan_gemv_bounded(M, N, K, group_size, slot->num_sms, vec_ok, kNoAllocScratchBytes,
                              &plan)) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "M=%lld N=%lld K=%lld needs more split-K scratch than the %zu-byte no-alloc array; "
             "use awq_gemm_f16 with a workspace",
             (long long)M, (long long)N, (long long)K, kNoAllocScratchBytes);
    return fail(AWQ_ERR_WORKSPACE, msg);
  }
  cudaError_t e = awq::launch_gemv(plan, x, ldx, qweight, qzeros, scales, out, ldo, (int)M,
                                   (int)N, (int)K, (int)group_size, slot->ptr,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(AWQ_ERR_CUDA, cudaGetErrorString(e));
  return AWQ_OK;
}
