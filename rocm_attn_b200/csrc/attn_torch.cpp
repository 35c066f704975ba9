// PyTorch binding of the sm_100a attention launcher, module
// `rocm_attn_ext`.  Mirrors the reference binding src/attn_torch.cpp:9-62 of
// JoursBleu/rocm_attn (same checks and messages, same argument meaning), with
// these changes: an optional softmax scale, inputs read through their strides
// instead of copied to contiguous tensors, the output from torch::empty (the
// kernel writes every element), the *current* stream of q's device, and a
// launcher status mapped to a Python RuntimeError.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <string>
#include <vector>

#include "attn_kernel.h"

namespace py = pybind11;

static const char* status_text(int s) {
  switch (s) {
    case ATTN_OK: return "ok";
    case ATTN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ATTN_ERR_UNSUPPORTED: return "unsupported dtype or head_dim (supported: float16/bfloat16/float32, 1 <= D <= 256)";
    case ATTN_ERR_MISALIGNED: return "q/k/v/out must be aligned to their element size";
    case ATTN_ERR_TENSOR_MAP: return "could not encode a TMA tensor map";
    case ATTN_ERR_LAUNCH: return "CUDA launch failed";
    case ATTN_ERR_DEVICE: return "the current device is not an sm_100 (B200-class) GPU";
    case ATTN_ERR_WATCHDOG: return "a kernel wait timed out; the output is invalid";
    default: return "unknown error";
  }
}

// One checked call: inputs read in place (or made contiguous), sizes, dtype,
// element strides over (batch, head, row) and the allocated output.
struct Prepared {
  torch::Tensor q, k, v, out;
  int64_t B, H, Sq, Skv, D;
  AttnDType dtype;
  long long qs[3], ks[3], vs[3];
};

// Reference: src/attn_torch.cpp:9-34 (checks, output allocation).
static Prepared prepare(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA/HIP tensor");
  TORCH_CHECK(k.is_cuda(), "k must be a CUDA/HIP tensor");
  TORCH_CHECK(v.is_cuda(), "v must be a CUDA/HIP tensor");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
              "q, k, v must have the same dtype");
  TORCH_CHECK(q.scalar_type() == torch::kFloat32 || q.scalar_type() == torch::kFloat16 ||
                  q.scalar_type() == torch::kBFloat16,
              "q, k, v must be float32, float16, or bfloat16");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q, k, v must be 4D [B, H, S, D]");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(), "q, k, v must be on the same device");

  Prepared c;
  // Inputs whose head dim is contiguous are read in place through their
  // strides (no copy, unlike the reference's .contiguous() calls); others are
  // made contiguous first.
  auto unit_inner = [](const torch::Tensor& t) { return t.dim() == 4 && (t.size(3) <= 1 || t.stride(3) == 1); };
  c.q = unit_inner(q) ? q : q.contiguous();
  c.k = unit_inner(k) ? k : k.contiguous();
  c.v = unit_inner(v) ? v : v.contiguous();

  c.B = c.q.size(0), c.H = c.q.size(1), c.Sq = c.q.size(2), c.D = c.q.size(3);
  c.Skv = c.k.size(2);
  TORCH_CHECK(c.k.size(0) == c.B && c.v.size(0) == c.B, "k/v batch size must match q");
  TORCH_CHECK(c.k.size(1) == c.H && c.v.size(1) == c.H, "k/v heads must match q");
  TORCH_CHECK(c.k.size(3) == c.D && c.v.size(3) == c.D, "k/v D must match q");
  TORCH_CHECK(c.v.size(2) == c.Skv, "k and v must have the same sequence length");
  TORCH_CHECK(c.B <= INT32_MAX && c.H <= INT32_MAX && c.Sq <= INT32_MAX && c.Skv <= INT32_MAX,
              "sizes must fit in 32-bit integers");

  c.out = torch::empty({c.B, c.H, c.Sq, c.D}, c.q.options());

  c.dtype = ATTN_F32;
  if (q.scalar_type() == torch::kFloat16) c.dtype = ATTN_F16;
  else if (q.scalar_type() == torch::kBFloat16) c.dtype = ATTN_BF16;

  // Strides over (batch, head, row).  A dim of size 1 may carry any stride in
  // torch; give it the contiguous one so TMA can take the tensor.
  auto strides3 = [](const torch::Tensor& t, long long* s) {
    s[2] = t.size(2) == 1 ? t.size(3) : t.stride(2);
    s[1] = t.size(1) == 1 ? s[2] * t.size(2) : t.stride(1);
    s[0] = t.size(0) == 1 ? s[1] * t.size(1) : t.stride(0);
  };
  strides3(c.q, c.qs);
  strides3(c.k, c.ks);
  strides3(c.v, c.vs);
  return c;
}

// Reference: src/attn_torch.cpp:9-57.
static torch::Tensor attn_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  Prepared c = prepare(q, k, v);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int st = launch_attn_forward_strided(c.q.data_ptr(), c.k.data_ptr(), c.v.data_ptr(), c.out.data_ptr(),
                                             static_cast<int>(c.B), static_cast<int>(c.H), static_cast<int>(c.Sq),
                                             static_cast<int>(c.Skv), static_cast<int>(c.D), causal,
                                             static_cast<float>(scale), c.dtype, c.qs, c.ks, c.vs, stream);
  TORCH_CHECK(st == ATTN_OK, "launch_attn_forward: ", status_text(st), " (status ", st, ")");
  return c.out;
}

// Several independent attention problems in one call (launch_attn_forward_batch):
// the same result per problem as attn_forward, with the tensor-core problems
// of one instantiation sharing a grid.  All problems share dtype, device,
// causal flag and scale.  No counterpart in the reference, whose benchmark
// calls the op once per shape (benchmark/bench_attention.py:81-100).
static std::vector<torch::Tensor> attn_forward_batch(std::vector<torch::Tensor> qs, std::vector<torch::Tensor> ks,
                                                     std::vector<torch::Tensor> vs, bool causal, double scale) {
  TORCH_CHECK(qs.size() == ks.size() && qs.size() == vs.size(), "q, k, v lists must have the same length");
  std::vector<torch::Tensor> outs;
  if (qs.empty()) return outs;
  const c10::cuda::CUDAGuard guard(qs[0].device());
  std::vector<Prepared> calls;
  calls.reserve(qs.size());
  for (size_t i = 0; i < qs.size(); ++i) {
    TORCH_CHECK(qs[i].device() == qs[0].device(), "all problems must be on the same device");
    TORCH_CHECK(qs[i].scalar_type() == qs[0].scalar_type(), "all problems must have the same dtype");
    calls.push_back(prepare(qs[i], ks[i], vs[i]));
  }
  std::vector<AttnProblem> probs(calls.size());
  for (size_t i = 0; i < calls.size(); ++i) {
    Prepared& c = calls[i];
    probs[i] = AttnProblem{c.q.data_ptr(), c.k.data_ptr(), c.v.data_ptr(), c.out.data_ptr(),
                           static_cast<int>(c.B), static_cast<int>(c.H), static_cast<int>(c.Sq),
                           static_cast<int>(c.Skv), static_cast<int>(c.D), causal, static_cast<float>(scale),
                           c.qs, c.ks, c.vs};
    outs.push_back(c.out);
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(qs[0].device().index()).stream();
  const int st = launch_attn_forward_batch(probs.data(), static_cast<int>(probs.size()), calls[0].dtype, stream);
  TORCH_CHECK(st == ATTN_OK, "launch_attn_forward_batch: ", status_text(st), " (status ", st, ")");
  return outs;
}

// Synchronises the current stream of `device` and returns (and clears) the
// kernel watchdog status: 0 when every earlier launch completed its waits.
static int check_status(int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(device)).stream();
  int status = 0;
  const int st = attn_get_status(stream, &status);
  TORCH_CHECK(st == ATTN_OK, "attn_get_status: ", status_text(st));
  return status;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("attn_forward", &attn_forward, "Fused attention forward (sm_100a tcgen05 kernel)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("causal") = false, py::arg("scale") = -1.0);
  m.def("attn_forward_batch", &attn_forward_batch,
        "Several independent attention problems in one call (grouped tcgen05 launches)", py::arg("qs"),
        py::arg("ks"), py::arg("vs"), py::arg("causal") = false, py::arg("scale") = -1.0);
  m.def("check_status", &check_status, "Read and clear the kernel watchdog status", py::arg("device") = 0);
  m.def("library_version", &attn_library_version);
  m.def("set_wait_limit_ns", [](uint64_t ns) { return static_cast<uint64_t>(attn_set_wait_limit_ns(ns)); },
        "Limit of each pipeline wait of the tensor-core kernel for later launches (0: default 2 s); returns the "
        "previous value. For tests of the watchdog path.",
        py::arg("ns"));
}
