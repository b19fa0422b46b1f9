// torch_ops.cpp -- the thin torch extension over the C ABI (include/rq_b200.h).
//
// Registers the layer's two entry points as torch operators,
//   torch.ops.rocm_qlora.linear_forward  (rq_linear_forward)
//   torch.ops.rocm_qlora.linear_dx       (rq_linear_dx)
// so that a QuantLinear / LoRALinear call goes from Python to the CUDA
// library through one dispatcher call: the output is allocated here, the
// launch goes to torch's current stream of the input's device, and a
// status other than RQ_OK raises with the library's message.  Nothing is
// computed here; the quantized weight arrives as its buffers plus the
// format (wfmt, N, K, block_size), as the C ABI takes it.  The Meta
// implementations give shapes to tracing (torch.compile, FakeTensor).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>

#include "../../include/rq_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return RQ_F32;
    case at::kBFloat16: return RQ_BF16;
    case at::kHalf: return RQ_F16;
    default: TORCH_CHECK(false, "rocm_qlora: unsupported dtype ", t);
  }
  return RQ_F32;
}

const void* ptr(const std::optional<at::Tensor>& t) { return t.has_value() && t->defined() ? t->data_ptr() : nullptr; }

void check(int rc, const char* what) {
  TORCH_CHECK(rc == RQ_OK, "rocm_qlora: ", what, " failed: ", rq_status_string(rc), " (status ", rc,
              rc == RQ_ERR_CUDA ? ", cuda error " + std::to_string(rq_last_cuda_error()) : std::string(), ")");
}

at::Tensor linear_forward(const at::Tensor& x, int64_t wfmt, const at::Tensor& q, const std::optional<at::Tensor>& scales,
                          const std::optional<at::Tensor>& c2, const std::optional<at::Tensor>& c2s, int64_t N,
                          int64_t K, int64_t block_size, const std::optional<at::Tensor>& lora_x,
                          const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& A,
                          const std::optional<at::Tensor>& B, double scaling, const at::Tensor& ws) {
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.size(1) == K, "rocm_qlora: x must be a contiguous [M, K] tensor");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0);
  const int r = A.has_value() && A->defined() ? (int)A->size(0) : 0;
  at::Tensor y = at::empty({M, N}, x.options());
  const cudaStream_t st = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const bool has_bias = bias.has_value() && bias->defined();
  const bool has_sc = scales.has_value() && scales->defined();
  check(rq_linear_forward((int)wfmt, q.data_ptr(), ptr(scales), has_sc ? dtype_code(scales->scalar_type()) : 0,
                          static_cast<const uint8_t*>(ptr(c2)), static_cast<const float*>(ptr(c2s)), N, K,
                          (int)block_size, x.data_ptr(), dtype_code(x.scalar_type()), M, ptr(lora_x), ptr(bias),
                          has_bias ? dtype_code(bias->scalar_type()) : 0, ptr(A), ptr(B), r, (float)scaling,
                          y.data_ptr(), ws.data_ptr(), ws.numel(), st),
        "rq_linear_forward");
  return y;
}

at::Tensor linear_dx(const at::Tensor& dy, int64_t wfmt, const at::Tensor& q, const std::optional<at::Tensor>& scales,
                     const std::optional<at::Tensor>& c2, const std::optional<at::Tensor>& c2s, int64_t N, int64_t K,
                     int64_t block_size, const std::optional<at::Tensor>& A, const std::optional<at::Tensor>& B,
                     double scaling, const at::Tensor& ws) {
  TORCH_CHECK(dy.dim() == 2 && dy.is_contiguous() && dy.size(1) == N, "rocm_qlora: dy must be a contiguous [M, N] tensor");
  const c10::cuda::CUDAGuard guard(dy.device());
  const int64_t M = dy.size(0);
  const int r = A.has_value() && A->defined() ? (int)A->size(0) : 0;
  at::Tensor dx = at::empty({M, K}, dy.options());
  const cudaStream_t st = c10::cuda::getCurrentCUDAStream(dy.device().index()).stream();
  const bool has_sc = scales.has_value() && scales->defined();
  check(rq_linear_dx((int)wfmt, q.data_ptr(), ptr(scales), has_sc ? dtype_code(scales->scalar_type()) : 0,
                     static_cast<const uint8_t*>(ptr(c2)), static_cast<const float*>(ptr(c2s)), N, K, (int)block_size,
                     dy.data_ptr(), dtype_code(dy.scalar_type()), M, ptr(A), ptr(B), r, (float)scaling, dx.data_ptr(),
                     ws.data_ptr(), ws.numel(), st),
        "rq_linear_dx");
  return dx;
}

at::Tensor linear_forward_meta(const at::Tensor& x, int64_t, const at::Tensor&, const std::optional<at::Tensor>&,
                               const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, int64_t N, int64_t,
                               int64_t, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                               const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, double,
                               const at::Tensor&) {
  return at::empty({x.size(0), N}, x.options());
}

at::Tensor linear_dx_meta(const at::Tensor& dy, int64_t, const at::Tensor&, const std::optional<at::Tensor>&,
                          const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, int64_t, int64_t K,
                          int64_t, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, double,
                          const at::Tensor&) {
  return at::empty({dy.size(0), K}, dy.options());
}

}  // namespace

TORCH_LIBRARY(rocm_qlora, m) {
  m.def(
      "linear_forward(Tensor x, int wfmt, Tensor q, Tensor? scales, Tensor? c2, Tensor? c2_scales, int N, int K, "
      "int block_size, Tensor? lora_x, Tensor? bias, Tensor? lora_a, Tensor? lora_b, float scaling, "
      "Tensor(a!) workspace) -> Tensor");
  m.def(
      "linear_dx(Tensor dy, int wfmt, Tensor q, Tensor? scales, Tensor? c2, Tensor? c2_scales, int N, int K, "
      "int block_size, Tensor? lora_a, Tensor? lora_b, float scaling, Tensor(a!) workspace) -> Tensor");
}

TORCH_LIBRARY_IMPL(rocm_qlora, CUDA, m) {
  m.impl("linear_forward", &linear_forward);
  m.impl("linear_dx", &linear_dx);
}

TORCH_LIBRARY_IMPL(rocm_qlora, Meta, m) {
  m.impl("linear_forward", &linear_forward_meta);
  m.impl("linear_dx", &linear_dx_meta);
}
