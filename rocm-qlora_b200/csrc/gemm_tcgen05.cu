// gemm_tcgen05.cu -- prefill/training-shaped fused dequant GEMM (tcgen05).
// (under construction: not yet selected by the dispatcher)
#include <cuda_runtime.h>

#include "rq_internal.h"

namespace rq {

bool gemm_supported(const LinearArgs& a, bool dx) {
  (void)a;
  (void)dx;
  return false;
}
int gemm_forward(const LinearArgs& a, const void* tdown, cudaStream_t st) {
  (void)a, (void)tdown, (void)st;
  return RQ_ERR_INVALID;
}
int gemm_dx(const LinearArgs& a, const void* gt, cudaStream_t st) {
  (void)a, (void)gt, (void)st;
  return RQ_ERR_INVALID;
}

}  // namespace rq
