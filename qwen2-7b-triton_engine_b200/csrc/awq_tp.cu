// awq_tp.cu -- tensor-parallel communicator of the fused row-parallel all-reduce
// (awq_tp_comm_* in include/awq_b200.h; the kernel side is the decode kernel's epilogue
// in awq_gemv_tma.cu, the entry point awq_gemm_f16_allreduce is in awq_capi.cu).
//
// Each rank owns one receive buffer (cudaMalloc, zeroed) and hands its CUDA IPC handle to
// the others; awq_tp_comm_open maps every other rank's buffer into this process (plain
// peer mappings over NVLink -- no multicast object, so a rank that dies leaves nothing
// bound on the others).  Buffers of ranks living in this same process are found in a
// process-local registry instead (CUDA IPC does not open a handle in its own process).
// Communicators made with max_rows > 0 also carry the planes of the prefill all-reduce
// (M > 16): the ranks' partial products are summed by row slice (each rank reads its
// slice from every rank over NVLink) and the sums gathered back through the other ranks'
// `res` planes -- tp_big_allreduce_kernel below; its layout is in awq_internal.h.
// The reference has no tensor parallelism (inference/engine.py:15).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/awq_b200.h"
#include "awq_common.cuh"
#include "awq_internal.h"

namespace {

std::mutex g_reg_mu;
std::map<std::string, void*>& registry() {   // IPC handle bytes -> buffer of this process
  static std::map<std::string, void*> r;
  return r;
}

int fail_tp(int code, const char* msg) { return awq::set_last_error(code, msg); }
int fail_tp_cuda(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  return awq::set_last_error(AWQ_ERR_CUDA, m.c_str());
}

}  // namespace

extern "C" {

int awq_tp_comm_create(int world, int rank, int64_t max_n, void* handle_out, awq_tp_comm** comm_out) {
  return awq_tp_comm_create_ex(world, rank, max_n, 0, handle_out, comm_out);
}

int awq_tp_comm_create_ex(int world, int rank, int64_t max_n, int64_t max_rows, void* handle_out,
                          awq_tp_comm** comm_out) {
  if (!comm_out || !handle_out) return fail_tp(AWQ_ERR_INVALID_ARG, "null handle_out or comm_out");
  *comm_out = nullptr;
  if (world < 1 || world > awq::kMaxWorld || rank < 0 || rank >= world)
    return fail_tp(AWQ_ERR_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
  if (max_n <= 0 || max_n % 8 || max_n > (int64_t)1 << 24)
    return fail_tp(AWQ_ERR_INVALID_ARG, "max_n must be a positive multiple of 8 below 2^24");
  if (max_rows < 0 || max_rows > (int64_t)1 << 20 || max_rows * max_n > (int64_t)1 << 32)
    return fail_tp(AWQ_ERR_INVALID_ARG, "max_rows must be 0..2^20 with max_rows * max_n <= 2^32");
  auto* c = new awq_tp_comm();
  cudaError_t e = cudaGetDevice(&c->device);
  if (e != cudaSuccess) { delete c; return fail_tp_cuda(e, "cudaGetDevice"); }
  c->world = world;
  c->rank = rank;
  c->max_n = max_n;
  c->max_rows = max_rows;
  c->max_tiles = 2 * (int)((max_n + 255) / 256);         // strips x up to 2 token chunks
  c->bytes = awq::tp_buffer_bytes(world, c->max_tiles);
  if (max_rows > 0)
    c->bytes = awq::tp_big_offset(world, c->max_tiles) + 2 * awq::tp_big_plane_bytes(max_rows, max_n);
  e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return fail_tp_cuda(e, "communicator buffer");
  }
  std::memcpy(handle_out, &h, AWQ_IPC_HANDLE_BYTES);
  {
    std::lock_guard<std::mutex> lock(g_reg_mu);
    registry()[std::string(reinterpret_cast<const char*>(&h), AWQ_IPC_HANDLE_BYTES)] = c->local;
  }
  c->peer[rank] = c->local;
  *comm_out = c;
  return AWQ_OK;
}

int awq_tp_comm_open(awq_tp_comm* c, const void* handles) {
  if (!c || !handles) return fail_tp(AWQ_ERR_INVALID_ARG, "null communicator or handles");
  if (c->ready) return fail_tp(AWQ_ERR_INVALID_ARG, "communicator already opened");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_tp_cuda(e, "cudaGetDevice");
  if (dev != c->device) return fail_tp(AWQ_ERR_INVALID_ARG, "current device is not the communicator's");
  const char* hb = static_cast<const char*>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    const std::string key(hb + (size_t)r * AWQ_IPC_HANDLE_BYTES, AWQ_IPC_HANDLE_BYTES);
    void* p = nullptr;
    {
      std::lock_guard<std::mutex> lock(g_reg_mu);
      auto it = registry().find(key);
      if (it != registry().end()) p = it->second;
    }
    if (!p) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, key.data(), AWQ_IPC_HANDLE_BYTES);
      e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        for (int q = 0; q < r; ++q)
          if (c->opened[q]) { cudaIpcCloseMemHandle(c->peer[q]); c->opened[q] = false; c->peer[q] = nullptr; }
        return fail_tp_cuda(e, "cudaIpcOpenMemHandle (is peer access over NVLink available?)");
      }
      c->opened[r] = true;
    }
    c->peer[r] = p;
  }
  c->ready = true;
  return AWQ_OK;
}

int awq_tp_comm_set_timeout(awq_tp_comm* c, uint64_t timeout_ns) {
  if (!c || timeout_ns == 0) return fail_tp(AWQ_ERR_INVALID_ARG, "null communicator or zero timeout");
  c->timeout_ns = timeout_ns;
  return AWQ_OK;
}

int awq_tp_comm_reset(awq_tp_comm* c) {
  if (!c || !c->ready) return fail_tp(AWQ_ERR_INVALID_ARG, "communicator missing or not opened");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_tp_cuda(e, "cudaGetDevice");
  if (dev != c->device) return fail_tp(AWQ_ERR_INVALID_ARG, "current device is not the communicator's");
  // every kernel of this device (this rank's fused calls included) must be finished
  // before the buffer is cleared; the caller keeps the other ranks out with a barrier
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail_tp_cuda(e, "communicator reset");
  return AWQ_OK;
}

int awq_tp_comm_destroy(awq_tp_comm* c) {
  if (!c) return AWQ_OK;
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) {
      cudaError_t e = cudaIpcCloseMemHandle(c->peer[r]);
      if (first == cudaSuccess) first = e;
    }
  {
    std::lock_guard<std::mutex> lock(g_reg_mu);
    for (auto it = registry().begin(); it != registry().end();)
      it = it->second == c->local ? registry().erase(it) : std::next(it);
  }
  if (c->local) {
    cudaError_t e = cudaFree(c->local);
    if (first == cudaSuccess) first = e;
  }
  delete c;
  return first == cudaSuccess ? AWQ_OK : fail_tp_cuda(first, "communicator teardown");
}

}  // extern "C"

namespace awq {

bool tp_ar_args(const awq_tp_comm* c, ArArgs* a) {
  if (!c || !c->ready) return false;
  *a = ArArgs{};
  a->world = c->world;
  a->rank = c->rank;
  a->max_tiles = c->max_tiles;
  for (int r = 0; r < c->world; ++r)
    a->data[r] = reinterpret_cast<unsigned long long*>(static_cast<char*>(c->peer[r]) +
                                                       tp_data_offset());
  a->state = static_cast<int*>(c->local);
  a->timeout_ns = c->timeout_ns;
  return true;
}

}  // namespace awq

namespace awq {
namespace {

struct BigArArgs {
  int world, rank, M, N;
  const __half* in[kMaxWorld];   // every rank's `in` plane (dense [M][N])
  __half* res[kMaxWorld];        // every rank's `res` plane
  unsigned* flags[kMaxWorld];    // every rank's flag words: in_flag[world], res_flag[world]
  int* state;                    // this rank's state words
  __half* out;
  int64_t ldo;
  unsigned long long timeout_ns;
  int* status;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits until flags f[0..n) reach `want` (a rank is never more than one call ahead, so
// "reached" is a wrap-safe >=), at most timeout_ns; on a time-out sets status bit 4 and
// returns: the call's output is then wrong, and every rank must reset the communicator.
__device__ void wait_flags(const unsigned* f, int n, unsigned want, unsigned long long timeout_ns,
                           int* status) {
  const unsigned long long t0 = timer_ns();
  for (int q = 0; q < n; ++q) {
    for (unsigned it = 0; (int)(ld_acquire_sys(f + q) - want) < 0; ++it) {
      if ((it & 63) == 63 && timer_ns() - t0 > timeout_ns) {
        atomicOr(status, kDevErrPeerTimeout);
        return;
      }
    }
  }
}

// One launch of num_sms CTAs (all resident together: small CTAs, no shared memory beyond
// two words), after the product kernel that wrote this rank's partial into its `in` plane.
//   1. CTA 0 publishes that partial (in_flag) to every rank; every CTA waits for all ranks'.
//   2. Reduce-scatter: this rank's row slice, summed over the ranks in rank order in fp32
//      (every rank's slice is summed by one rank only, so all ranks get the same bits),
//      rounded to fp16 and stored into every rank's `res` plane.  The last CTA to finish
//      publishes the slice (res_flag) to every rank.
//   3. All-gather: once every slice is in, the `res` plane is copied into out.
// A plane is rewritten only after every rank has read it: a rank's next partial starts
// after its own step 3, which needs every rank's step 2, which needs every rank's reads.
constexpr int kArUnroll = 4;   // 16-byte vectors per thread and round, loads issued together

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__global__ void __launch_bounds__(256) tp_big_allreduce_kernel(const BigArArgs a) {
  __shared__ unsigned s_flag;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  // launched as a programmatic dependent of the product kernel: nothing is read before
  // that kernel has completed and its writes are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) s_flag = (unsigned)*reinterpret_cast<volatile int*>(a.state) + 1u;
  __syncthreads();
  const unsigned flag = s_flag;
  const unsigned* mine = a.flags[a.rank];
  if (blockIdx.x == 0 && tid < a.world) {
    fence_acq_rel_sys();
    st_release_sys(a.flags[tid] + a.rank, flag);
  }
  if (tid == 0) wait_flags(mine, a.world, flag, a.timeout_ns, a.status);
  __syncthreads();

  const int64_t r0 = (int64_t)a.M * a.rank / a.world, r1 = (int64_t)a.M * (a.rank + 1) / a.world;
  const int64_t nv = (r1 - r0) * a.N / 8, base = r0 * a.N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + tid; v0 < nv; v0 += stride * kArUnroll) {
    float acc[kArUnroll][8];
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
    for (int q = 0; q < a.world; ++q) {           // rank order
      uint4 ld[kArUnroll];
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) {
        const int64_t v = v0 + u * stride;
        ld[u] = v < nv ? __ldcg(reinterpret_cast<const uint4*>(a.in[q] + base + v * 8))
                       : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) {
        const uint32_t w[4] = {ld[u].x, ld[u].y, ld[u].z, ld[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(u32_as_h2(w[i]));
          acc[u][2 * i] += f.x;
          acc[u][2 * i + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      if (v >= nv) continue;
      uint4 o;
      o.x = h2_as_u32(__floats2half2_rn(acc[u][0], acc[u][1]));
      o.y = h2_as_u32(__floats2half2_rn(acc[u][2], acc[u][3]));
      o.z = h2_as_u32(__floats2half2_rn(acc[u][4], acc[u][5]));
      o.w = h2_as_u32(__floats2half2_rn(acc[u][6], acc[u][7]));
      for (int q = 0; q < a.world; ++q) *reinterpret_cast<uint4*>(a.res[q] + base + v * 8) = o;
    }
  }
  // the CTA's slice stores (ordered by the barrier), then its count; the last CTA
  // publishes the slice to every rank
  __syncthreads();
  if (tid == 0) {
    fence_acq_rel_sys();
    s_last = atomicAdd(a.state + 1, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (tid == 0) a.state[1] = 0;
    if (tid < a.world) {
      fence_acq_rel_sys();
      st_release_sys(a.flags[tid] + a.world + a.rank, flag);
    }
  }
  if (tid == 0) wait_flags(mine + a.world, a.world, flag, a.timeout_ns, a.status);
  __syncthreads();

  const int64_t tv = (int64_t)a.M * a.N / 8;
  const int vpr = a.N / 8;
  for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + tid; v0 < tv; v0 += stride * kArUnroll) {
    uint4 ld[kArUnroll];
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      ld[u] = v < tv ? __ldcg(reinterpret_cast<const uint4*>(a.res[a.rank] + v * 8))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      if (v >= tv) continue;
      const int64_t row = v / vpr, col = (v - row * vpr) * 8;
      *reinterpret_cast<uint4*>(a.out + row * a.ldo + col) = ld[u];
    }
  }
  __syncthreads();
  if (tid == 0 && atomicAdd(a.state + 2, 1) == (int)gridDim.x - 1) {
    a.state[2] = 0;
    a.state[0] = (int)flag;    // calls so far: the next call publishes flag + 1
  }
}

}  // namespace

void* tp_big_in_plane(const awq_tp_comm* c) {
  if (!c || !c->ready || c->max_rows <= 0) return nullptr;
  return static_cast<char*>(c->local) + tp_big_offset(c->world, c->max_tiles);
}

cudaError_t launch_tp_big_allreduce(const awq_tp_comm* c, int M, int N, void* out, int64_t ldo,
                                    int num_sms, int* dev_status, cudaStream_t stream) {
  if (!c || !c->ready || c->max_rows < M || N > c->max_n || N % 8 || M < 1 || ldo % 8 ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  BigArArgs a = {};
  a.world = c->world;
  a.rank = c->rank;
  a.M = M;
  a.N = N;
  const size_t off = tp_big_offset(c->world, c->max_tiles);
  const size_t plane = tp_big_plane_bytes(c->max_rows, c->max_n);
  for (int r = 0; r < c->world; ++r) {
    char* b = static_cast<char*>(c->peer[r]);
    a.in[r] = reinterpret_cast<const __half*>(b + off);
    a.res[r] = reinterpret_cast<__half*>(b + off + plane);
    a.flags[r] = reinterpret_cast<unsigned*>(b + kBigFlagOffset);
  }
  a.state = reinterpret_cast<int*>(static_cast<char*>(c->local) + kBigStateOffset);
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.timeout_ns = c->timeout_ns;
  a.status = dev_status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tp_big_allreduce_kernel, a);
}

}  // namespace awq
