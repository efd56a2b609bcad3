// awq_torch_ext.cpp -- the PyTorch-facing host glue of the drop-in, in C++.
//
// kernels.awq_gemm.awq_gemm_forward (songqiuyu/Qwen2-7B-Triton_Engine kernels/awq_gemm.py:
// 237-284) runs once per linear layer per decode step, so its host cost is paid 112 times
// per token of Qwen2-7B.  This module does the per-call work of awq_b200.gemm --
// argument checks, the output allocation, the current stream, the per-(device, stream)
// split-K workspace -- in C++ and calls the library through its C ABI
// (include/awq_b200.h; no torch types cross that boundary).  The Python package uses it
// when it is built and keeps its ctypes path otherwise; both call the same entry points.
//
// Errors: the same exception types as the Python path -- TypeError for dtypes,
// ValueError for shapes, devices and CPU tensors ("... CUDA only ..."), and the
// package's AwqError (registered by set_error_class) for a non-zero return code.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <tuple>

#include "../../include/awq_b200.h"

namespace {

PyObject* g_error_class = nullptr;   // awq_b200._lib.AwqError

[[noreturn]] void raise_awq(int rc) {
  const char* msg = awq_last_error();
  if (g_error_class) {
    PyObject* exc = PyObject_CallFunction(g_error_class, "is", rc, msg ? msg : "");
    if (exc) {
      PyErr_SetObject(g_error_class, exc);
      Py_DECREF(exc);
    }
    throw pybind11::error_already_set();
  }
  TORCH_CHECK(false, "libawq_b200 error ", rc, ": ", msg ? msg : "");
}

void require_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda(), name, " is on ", t.device().str(),
                    "; the AWQ kernels run on CUDA only (no CPU fallback)");
}

// Contiguous and 16-byte aligned (copies only when needed).
at::Tensor dense16(const at::Tensor& t) {
  at::Tensor r = t.is_contiguous() ? t : t.contiguous();
  if (reinterpret_cast<uintptr_t>(r.data_ptr()) % 16) r = r.clone();
  return r;
}

// Validates the packed layout (model/qwen2.py:34-36); returns (K, N) with N =
// scales.shape[1] as in awq_gemm_forward (kernels/awq_gemm.py:247).
std::pair<int64_t, int64_t> check_weights(const at::Tensor& qw, const at::Tensor& qz,
                                          const at::Tensor& s, int64_t gs) {
  require_cuda(qw, "qweight");
  require_cuda(qz, "qzeros");
  require_cuda(s, "scales");
  TORCH_CHECK_VALUE(qw.dim() == 2 && qz.dim() == 2 && s.dim() == 2,
                    "qweight, qzeros and scales must be 2-D");
  TORCH_CHECK_TYPE(qw.scalar_type() == at::kInt && qz.scalar_type() == at::kInt,
                   "qweight and qzeros must be int32");
  TORCH_CHECK_TYPE(s.scalar_type() == at::kHalf, "scales must be float16");
  TORCH_CHECK_VALUE(qw.device() == qz.device() && qw.device() == s.device(),
                    "qweight, qzeros and scales must be on one device");
  const int64_t K = qw.size(0), N = s.size(1);
  TORCH_CHECK_VALUE(qw.size(1) * 8 == N, "scales.shape[1]=", N, " but qweight packs ",
                    qw.size(1) * 8, " columns");
  TORCH_CHECK_VALUE(gs > 0 && K % gs == 0, "K=", K, " is not a multiple of group_size=", gs);
  const int64_t G = K / gs;
  TORCH_CHECK_VALUE(qz.size(0) == G && qz.size(1) == N / 8 && s.size(0) == G,
                    "qzeros / scales do not match [K/group_size=", G, ", N/8=", N / 8, "] / [",
                    G, ", ", N, "]");
  return {K, N};
}

// Zero-initialised split-K workspace per (device, stream), grown on demand.  The kernels
// leave its counters at zero after every call, so it is zeroed once per allocation.
std::mutex g_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor> g_ws;
std::map<std::tuple<int, int64_t, int64_t, int64_t, int64_t, bool>, size_t> g_need;

size_t workspace_need(int dev, int64_t M, int64_t N, int64_t K, int64_t gs, bool silu) {
  const auto key = std::make_tuple(dev, M, N, K, gs, silu);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_need.find(key);
    if (it != g_need.end()) return it->second;
  }
  const size_t need = silu ? awq_gemm_silu_mul_workspace_bytes(M, N, K, gs)
                           : awq_gemm_workspace_bytes(M, N, K, gs);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_need.size() > 65536) g_need.clear();
  g_need[key] = need;
  return need;
}

at::Tensor workspace_for(const at::Device& dev, cudaStream_t st, size_t need) {
  std::lock_guard<std::mutex> lk(g_mu);
  at::Tensor& ws = g_ws[{dev.index(), st}];
  if (!ws.defined() || (size_t)ws.numel() < need) {
    const int64_t size = need > (size_t)(1 << 20) ? (int64_t)need : (int64_t)(1 << 20);
    ws = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return ws;
}

// The product behind gemm / forward: out fp16 [M, N] (or [M, N/2] with silu) on the
// current stream.
at::Tensor gemm_impl(at::Tensor x, at::Tensor qw, at::Tensor qz, at::Tensor s, int64_t gs,
                     int64_t path, c10::optional<at::Tensor> out_opt,
                     c10::optional<at::Tensor> bias_opt, bool silu) {
  auto [K, N] = check_weights(qw, qz, s, gs);
  qw = dense16(qw);
  qz = dense16(qz);
  s = dense16(s);
  require_cuda(x, "x");
  TORCH_CHECK_TYPE(x.scalar_type() == at::kHalf, "x must be float16, got ", x.scalar_type());
  TORCH_CHECK_VALUE(x.dim() == 2 && x.size(1) == K, "x must be [M, K=", K, "], got ", x.sizes());
  TORCH_CHECK_VALUE(x.device() == qw.device(), "x and the weights must be on one device");
  if (silu) TORCH_CHECK_VALUE(N % 2 == 0, "N=", N, " is not even: no gate / up halves");
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = *bias_opt;
    require_cuda(bias, "bias");
    TORCH_CHECK_VALUE(bias.scalar_type() == at::kHalf && bias.dim() == 1 && bias.size(0) == N,
                      "bias must be float16 [N=", N, "]");
    TORCH_CHECK_VALUE(path == AWQ_PATH_AUTO, "the bias epilogue runs on the automatic kernel choice only");
    bias = bias.contiguous();
  }
  const int64_t M = x.size(0);
  const int64_t NO = silu ? N / 2 : N;
  at::Tensor out = out_opt.has_value() && out_opt->defined()
                       ? *out_opt
                       : at::empty({M, NO}, x.options());
  if (M == 0) return out;
  if (x.stride(1) != 1 || reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 || (x.stride(0) * 2) % 16) {
    x = x.contiguous();
    if (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) x = x.clone();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const size_t need = workspace_need(x.device().index(), M, N, K, gs, silu);
  at::Tensor ws;
  if (need) ws = workspace_for(x.device(), st, need);
  void* wsp = ws.defined() ? ws.data_ptr() : nullptr;
  const size_t wsn = ws.defined() ? (size_t)ws.numel() : 0;
  int rc;
  if (silu) {
    rc = awq_gemm_f16_silu_mul(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qz.data_ptr<int32_t>(),
                               s.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs, wsp, wsn, st);
  } else if (bias.defined()) {
    rc = awq_gemm_f16_bias(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qz.data_ptr<int32_t>(),
                           s.data_ptr(), bias.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs,
                           wsp, wsn, st);
  } else {
    rc = awq_gemm_f16_ex(x.data_ptr(), x.stride(0), qw.data_ptr<int32_t>(), qz.data_ptr<int32_t>(),
                         s.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs, wsp, wsn, st,
                         (int)path);
  }
  if (rc != AWQ_OK) raise_awq(rc);
  return out;
}

// awq_gemm_forward's shape handling (kernels/awq_gemm.py:244-284): x [..., K] -> [..., N].
at::Tensor forward_impl(const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz,
                        const at::Tensor& s, int64_t gs, c10::optional<at::Tensor> bias, bool silu) {
  TORCH_CHECK_VALUE(x.dim() >= 1, "x must have at least one dimension");
  const int64_t N = s.dim() == 2 ? s.size(1) : 0;
  at::Tensor out = gemm_impl(x.reshape({-1, x.size(-1)}), qw, qz, s, gs, AWQ_PATH_AUTO,
                             c10::nullopt, bias, silu);
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end() - 1);
  shape.push_back(silu ? N / 2 : N);
  return out.view(shape);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ host glue of the AWQ drop-in (calls libawq_b200 through its C ABI)";
  m.def("set_error_class", [](pybind11::object cls) {
    Py_XDECREF(g_error_class);
    g_error_class = cls.ptr();
    Py_INCREF(g_error_class);
  });
  m.def("gemm", [](at::Tensor x, at::Tensor qw, at::Tensor qz, at::Tensor s, int64_t gs, int64_t path,
                   c10::optional<at::Tensor> out, c10::optional<at::Tensor> bias) {
          return gemm_impl(x, qw, qz, s, gs, path, out, bias, false);
        });
  m.def("gemm_silu_mul", [](at::Tensor x, at::Tensor qw, at::Tensor qz, at::Tensor s, int64_t gs,
                            c10::optional<at::Tensor> out) {
          return gemm_impl(x, qw, qz, s, gs, AWQ_PATH_AUTO, out, c10::nullopt, true);
        });
  m.def("forward", [](const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz,
                      const at::Tensor& s, int64_t gs) {
          return forward_impl(x, qw, qz, s, gs, c10::nullopt, false);
        });
  m.def("forward_bias", [](const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz,
                           const at::Tensor& s, const at::Tensor& bias, int64_t gs) {
          return forward_impl(x, qw, qz, s, gs, bias, false);
        });
  m.def("forward_silu_mul", [](const at::Tensor& x, const at::Tensor& qw, const at::Tensor& qz,
                               const at::Tensor& s, int64_t gs) {
          return forward_impl(x, qw, qz, s, gs, c10::nullopt, true);
        });
}
