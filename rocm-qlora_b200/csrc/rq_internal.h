// rq_internal.h -- internal (C++) interface between the C-ABI layer and the
// kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rq_b200.h"

namespace rq {

// Kernel family of the last layer call in this thread (RQ_PATH_*).
int last_path();

// Decode GEMV numerics (rq_set_decode_exact; gemv_nf4.cu).
void set_decode_exact(int on);

// Records the CUDA error of the last failing launch in this thread.
void set_cuda_error(cudaError_t e);

// Driver-API failures (tensor-map encoding) are recorded as this base plus
// the CUresult, so that they do not read as runtime error codes.
constexpr int kDriverErrorBase = 10000;

// Raises a kernel's dynamic shared memory limit to `bytes` on the current
// device (once per kernel, device and size; thread-safe).
int ensure_smem_limit(const void* kernel, size_t bytes);

// Maps the launch status of the kernel just issued to an RQ_* status.
inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return RQ_OK;
}

int nf4_quantize(const void* x, int dtype, int64_t n, int bs, uint8_t* packed, void* scales, cudaStream_t st);
int nf4_dequantize(const uint8_t* p, int64_t nbytes, const void* s, int sdt, int bs, void* out, int odt,
                   cudaStream_t st);
int dq_dequantize(const uint8_t* p, int64_t numel, const uint8_t* c2, const float* c2s, int fp8, int bs, int bs2,
                  void* out, int odt, cudaStream_t st);
int dq_quantize_scales(const float* c1, int64_t nb, int bs2, int fp8, uint8_t* c2, float* c2s, cudaStream_t st);
int int8_quantize(const void* x, int dtype, int64_t n, int bs, int8_t* q, void* scales, cudaStream_t st);
int int8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t cols, int8_t* q, void* scales,
                       cudaStream_t st);
int int8_dequantize(const int8_t* q, int64_t n, const void* s, int sdt, int bs, int64_t cols, void* out, int odt,
                    cudaStream_t st);

__host__ __device__ inline bool is_nf4_fmt(int fmt) {
  return fmt == RQ_W_NF4 || fmt == RQ_W_NF4_DQ_FP8 || fmt == RQ_W_NF4_DQ_INT8;
}

// Weight operand of a quantized linear layer, as the kernels see it.
struct QWeight {
  int fmt;              // RQ_W_*
  const void* q;        // NF4 packed codes or int8 values
  const void* scales;   // per-block / per-row scales (non-DQ formats)
  int sdt;              // dtype of `scales`
  const uint8_t* c2;    // DQ second-level codes
  const float* c2s;     // DQ second-level scales
  int64_t N, K;
  int bs;               // first-level block size
};

struct LinearArgs {
  QWeight w;
  const void* x;        // [M, K] (forward) or dy [M, N] (dx)
  const void* lora_x;   // input of the adapter branch (forward), usually x
  int xdt;
  int64_t M;
  const void* bias;
  int bdt;
  const void* lora_a;   // [r, K]
  const void* lora_b;   // [N, r]
  int r;
  float scaling;
  void* y;              // [M, N] (forward) or dx [M, K]
  void* ws;
  int64_t ws_bytes;
  const RqGather* gather;  // forward only: write the output into every rank's Y (nullptr: local y)
};

// kernel families (linear.cu picks one per call)
int lora_down(int dt, bool w_transposed, const void* X, int64_t M, int64_t Kr, const void* W2, int R, float pre_s,
              bool do_pre, void* out, float* partial, int64_t partial_elems, unsigned* counters, int ncounters,
              cudaStream_t st);
int simt_forward(const LinearArgs& a, const void* tdown, cudaStream_t st);
int simt_dx(const LinearArgs& a, const void* gt, cudaStream_t st);
bool gemv_supported(const LinearArgs& a);
bool gemv_fuse_down(const LinearArgs& a);
// `partial` / `counters` (workspace): the NF4 GEMV computes tdown itself
int gemv_forward(const LinearArgs& a, const void* tdown, cudaStream_t st, float* partial = nullptr,
                 unsigned* counters = nullptr);

int linear_forward(const LinearArgs& a, cudaStream_t st);
int weight_absmax(const QWeight& w, int dt, float* out, cudaStream_t st);
int weight_to_fp8(const QWeight& w, int dt, float s, uint8_t* out, cudaStream_t st);
int merge_weight(const QWeight& w, const float* A, const float* B, int r, float s, int mode, void* out, int odt,
                 cudaStream_t st);
int linear_dx(const LinearArgs& a, cudaStream_t st);
int64_t linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int r);

}  // namespace rq
