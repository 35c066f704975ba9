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

// Reference: src/attn_torch.cpp:9-57.
static torch::Tensor attn_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale) {
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

  const c10::cuda::CUDAGuard guard(q.device());
  // Inputs whose head dim is contiguous are read in place through their
  // strides (no copy, unlike the reference's .contiguous() calls); others are
  // made contiguous first.
  auto unit_inner = [](const torch::Tensor& t) { return t.dim() == 4 && (t.size(3) <= 1 || t.stride(3) == 1); };
  auto q_c = unit_inner(q) ? q : q.contiguous();
  auto k_c = unit_inner(k) ? k : k.contiguous();
  auto v_c = unit_inner(v) ? v : v.contiguous();

  const int64_t B = q_c.size(0), H = q_c.size(1), Sq = q_c.size(2), D = q_c.size(3);
  const int64_t Skv = k_c.size(2);
  TORCH_CHECK(k_c.size(0) == B && v_c.size(0) == B, "k/v batch size must match q");
  TORCH_CHECK(k_c.size(1) == H && v_c.size(1) == H, "k/v heads must match q");
  TORCH_CHECK(k_c.size(3) == D && v_c.size(3) == D, "k/v D must match q");
  TORCH_CHECK(v_c.size(2) == Skv, "k and v must have the same sequence length");
  TORCH_CHECK(B <= INT32_MAX && H <= INT32_MAX && Sq <= INT32_MAX && Skv <= INT32_MAX,
              "sizes must fit in 32-bit integers");

  auto out = torch::empty({B, H, Sq, D}, q_c.options());

  AttnDType dtype = ATTN_F32;
  if (q.scalar_type() == torch::kFloat16) dtype = ATTN_F16;
  else if (q.scalar_type() == torch::kBFloat16) dtype = ATTN_BF16;

  cudaStream_t stream = at::cuda::getCurrentCUDAStream(q.device().index()).stream();
  // Strides over (batch, head, row).  A dim of size 1 may carry any stride in
  // torch; give it the contiguous one so TMA can take the tensor.
  auto strides3 = [](const torch::Tensor& t, long long* s) {
    s[2] = t.size(2) == 1 ? t.size(3) : t.stride(2);
    s[1] = t.size(1) == 1 ? s[2] * t.size(2) : t.stride(1);
    s[0] = t.size(0) == 1 ? s[1] * t.size(1) : t.stride(0);
  };
  long long qs[3], ks[3], vs[3];
  strides3(q_c, qs);
  strides3(k_c, ks);
  strides3(v_c, vs);
  const int st = launch_attn_forward_strided(q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), out.data_ptr(),
                                             static_cast<int>(B), static_cast<int>(H), static_cast<int>(Sq),
                                             static_cast<int>(Skv), static_cast<int>(D), causal,
                                             static_cast<float>(scale), dtype, qs, ks, vs, stream);
  TORCH_CHECK(st == ATTN_OK, "launch_attn_forward: ", status_text(st), " (status ", st, ")");
  return out;
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
  m.def("check_status", &check_status, "Read and clear the kernel watchdog status", py::arg("device") = 0);
  m.def("library_version", &attn_library_version);
  m.def("set_wait_limit_ns", [](uint64_t ns) { return static_cast<uint64_t>(attn_set_wait_limit_ns(ns)); },
        "Limit of each pipeline wait of the tensor-core kernel for later launches (0: default 2 s); returns the "
        "previous value. For tests of the watchdog path.",
        py::arg("ns"));
}
