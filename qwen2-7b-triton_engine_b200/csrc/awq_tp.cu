// awq_tp.cu -- tensor-parallel communicator of the fused row-parallel all-reduce
// (awq_tp_comm_* in include/awq_b200.h; the kernel side is the decode kernel's epilogue
// in awq_gemv_tma.cu, the entry point awq_gemm_f16_allreduce is in awq_capi.cu).
//
// Each rank owns one receive buffer (cudaMalloc, zeroed) and hands its CUDA IPC handle to
// the others; awq_tp_comm_open maps every other rank's buffer into this process (plain
// peer mappings over NVLink -- no multicast object, so a rank that dies leaves nothing
// bound on the others).  Buffers of ranks living in this same process are found in a
// process-local registry instead (CUDA IPC does not open a handle in its own process).
// The reference has no tensor parallelism (inference/engine.py:15).
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/awq_b200.h"
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
  if (!comm_out || !handle_out) return fail_tp(AWQ_ERR_INVALID_ARG, "null handle_out or comm_out");
  *comm_out = nullptr;
  if (world < 1 || world > awq::kMaxWorld || rank < 0 || rank >= world)
    return fail_tp(AWQ_ERR_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
  if (max_n <= 0 || max_n % 8 || max_n > (int64_t)1 << 24)
    return fail_tp(AWQ_ERR_INVALID_ARG, "max_n must be a positive multiple of 8 below 2^24");
  auto* c = new awq_tp_comm();
  cudaError_t e = cudaGetDevice(&c->device);
  if (e != cudaSuccess) { delete c; return fail_tp_cuda(e, "cudaGetDevice"); }
  c->world = world;
  c->rank = rank;
  c->max_n = max_n;
  c->max_tiles = 2 * (int)((max_n + 255) / 256);         // strips x up to 2 token chunks
  c->bytes = awq::tp_buffer_bytes(world, c->max_tiles);
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
