// peer.cu -- device memory shared between the ranks of one node (CUDA IPC
// over NVLink), and the C entry point of the column-sharded layer whose
// output every rank writes into every rank's Y (the gather is fused into
// the decode GEMV's epilogue, gemv_nf4.cu).
#include <cuda_runtime.h>
#include <string.h>

#include "rq_internal.h"

namespace rq {
namespace {
int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return RQ_OK;
  set_cuda_error(e);
  return RQ_ERR_CUDA;
}
}  // namespace
}  // namespace rq

extern "C" {

int rq_peer_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return RQ_ERR_INVALID;
  *ptr = nullptr;
  void* p = nullptr;
  int rc = rq::cuda_status(cudaMalloc(&p, (size_t)bytes));
  if (rc != RQ_OK) return rc;
  rc = rq::cuda_status(cudaMemset(p, 0, (size_t)bytes));
  if (rc != RQ_OK) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return RQ_OK;
}

int rq_peer_free(void* ptr) { return ptr ? rq::cuda_status(cudaFree(ptr)) : RQ_OK; }

int rq_peer_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return RQ_ERR_INVALID;
  cudaIpcMemHandle_t h;
  const int rc = rq::cuda_status(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  if (rc != RQ_OK) return rc;
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return RQ_OK;
}

int rq_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return RQ_ERR_INVALID;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return rq::cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int rq_peer_close(void* ptr) { return ptr ? rq::cuda_status(cudaIpcCloseMemHandle(ptr)) : RQ_OK; }

}  // extern "C"
