// capi.cu -- the extern "C" boundary (include/rq_b200.h).
//
// Every entry point validates its arguments on the host, checks that the
// current device is an sm_100 part, and then launches on the caller's
// stream.  Nothing here allocates device memory.
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "rq_internal.h"

namespace rq {

static thread_local int g_last_cuda_error = 0;
static thread_local int g_last_status = 0;

void set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

int ensure_smem_limit(const void* kernel, size_t bytes) {
  struct Entry {
    const void* k;
    int dev;
    size_t bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : done)
    if (e.k == kernel && e.dev == dev && e.bytes >= bytes) return RQ_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  done.push_back({kernel, dev, bytes});
  return RQ_OK;
}

static int device_ok() {
  static int cache[64];  // 0 unknown, 1 ok, -1 not sm_100
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return RQ_ERR_DEVICE;
  if (cache[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cache[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  return cache[dev] == 1 ? RQ_OK : RQ_ERR_DEVICE;
}

static bool dtype_ok(int dt) { return dt == RQ_F32 || dt == RQ_BF16 || dt == RQ_F16; }

static int dtype_size(int dt) { return dt == RQ_F32 ? 4 : 2; }

static int check_weight(int wfmt, const void* q, const void* scales, int sdt, const uint8_t* c2, const float* c2s,
                        int64_t N, int64_t K, int bs) {
  if (N < 0 || K < 0 || !q) return RQ_ERR_INVALID;
  if (wfmt < RQ_W_NF4 || wfmt > RQ_W_INT8_ROW) return RQ_ERR_DTYPE;
  if (wfmt == RQ_W_NF4_DQ_FP8 || wfmt == RQ_W_NF4_DQ_INT8) {
    if (!c2 || !c2s) return RQ_ERR_INVALID;
  } else {
    if (!scales || !dtype_ok(sdt)) return RQ_ERR_INVALID;
  }
  if (wfmt != RQ_W_INT8_ROW && (bs < 2 || (is_nf4_fmt(wfmt) && (bs & 1)))) return RQ_ERR_INVALID;
  return RQ_OK;
}

static int fill_args(LinearArgs* a, int wfmt, const void* q, const void* scales, int sdt, const uint8_t* c2,
                     const float* c2s, int64_t N, int64_t K, int bs, const void* x, int xdt, int64_t M,
                     const void* bias, int bdt, const void* la, const void* lb, int r, float scaling, void* y,
                     void* ws, int64_t ws_bytes) {
  int rc = check_weight(wfmt, q, scales, sdt, c2, c2s, N, K, bs);
  if (rc != RQ_OK) return rc;
  if (!dtype_ok(xdt)) return RQ_ERR_DTYPE;
  if (M < 0 || (M > 0 && (!x || !y))) return RQ_ERR_INVALID;
  if (bias && !dtype_ok(bdt)) return RQ_ERR_DTYPE;
  if (r < 0 || r > 128) return RQ_ERR_INVALID;
  if (r > 0 && (!la || !lb)) return RQ_ERR_INVALID;
  if ((uintptr_t)x % dtype_size(xdt) || (uintptr_t)y % dtype_size(xdt)) return RQ_ERR_ALIGN;
  a->w = QWeight{wfmt, q, scales, sdt, c2, c2s, N, K, bs};
  a->x = x;
  a->xdt = xdt;
  a->M = M;
  a->bias = bias;
  a->bdt = bdt;
  a->lora_a = la;
  a->lora_b = lb;
  a->r = r;
  a->scaling = scaling;
  a->y = y;
  a->ws = ws;
  a->ws_bytes = ws_bytes;
  a->lora_x = x;
  a->gather = nullptr;
  return RQ_OK;
}

}  // namespace rq

using namespace rq;

#define RQ_PROLOGUE()               \
  do {                              \
    int _rc = device_ok();          \
    if (_rc != RQ_OK) return _rc;   \
  } while (0)

extern "C" {

int rq_abi_version(void) { return 3; }

const char* rq_status_string(int s) {
  switch (s) {
    case RQ_OK: return "ok";
    case RQ_ERR_INVALID: return "invalid argument";
    case RQ_ERR_ALIGN: return "misaligned pointer";
    case RQ_ERR_DTYPE: return "unsupported dtype or format";
    case RQ_ERR_CUDA: return "CUDA error";
    case RQ_ERR_WORKSPACE: return "workspace missing or too small";
    case RQ_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case RQ_ERR_SCRATCH: return "request exceeds the built-in scratch of rq_linear_forward_noalloc";
  }
  return "unknown status";
}

int rq_last_cuda_error(void) { return g_last_cuda_error; }
int rq_last_status(void) { return g_last_status; }
int rq_last_path(void) { return rq::last_path(); }
void rq_set_decode_exact(int exact) { rq::set_decode_exact(exact); }

int rq_nf4_quantize(const void* x, int dtype, int64_t numel, int block_size, uint8_t* packed, void* scales,
                    void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(dtype)) return RQ_ERR_DTYPE;
  if (numel < 0 || block_size < 2 || (block_size & 1)) return RQ_ERR_INVALID;
  if (numel == 0) return RQ_OK;
  if (!x || !packed || !scales) return RQ_ERR_INVALID;
  if ((uintptr_t)x % dtype_size(dtype) || (uintptr_t)scales % dtype_size(dtype)) return RQ_ERR_ALIGN;
  return nf4_quantize(x, dtype, numel, block_size, packed, scales, (cudaStream_t)stream);
}

int rq_nf4_dequantize(const uint8_t* packed, int64_t nbytes, const void* scales, int scale_dtype, int block_size,
                      void* out, int out_dtype, void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(scale_dtype) || !dtype_ok(out_dtype)) return RQ_ERR_DTYPE;
  if (nbytes < 0 || block_size < 2 || (block_size & 1)) return RQ_ERR_INVALID;
  if (nbytes == 0) return RQ_OK;
  if (!packed || !scales || !out) return RQ_ERR_INVALID;
  if ((uintptr_t)out % dtype_size(out_dtype) || (uintptr_t)scales % dtype_size(scale_dtype)) return RQ_ERR_ALIGN;
  return nf4_dequantize(packed, nbytes, scales, scale_dtype, block_size, out, out_dtype, (cudaStream_t)stream);
}

int rq_int8_quantize(const void* x, int dtype, int64_t numel, int block_size, int8_t* q, void* scales,
                     void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(dtype)) return RQ_ERR_DTYPE;
  if (numel < 0 || block_size < 1) return RQ_ERR_INVALID;
  if (numel == 0) return RQ_OK;
  if (!x || !q || !scales) return RQ_ERR_INVALID;
  if ((uintptr_t)x % dtype_size(dtype) || (uintptr_t)scales % dtype_size(dtype)) return RQ_ERR_ALIGN;
  return int8_quantize(x, dtype, numel, block_size, q, scales, (cudaStream_t)stream);
}

int rq_int8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t cols, int8_t* q, void* scales,
                          void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(dtype)) return RQ_ERR_DTYPE;
  if (rows < 0 || cols < 0) return RQ_ERR_INVALID;
  if (rows == 0) return RQ_OK;
  if (!x || !q || !scales) return RQ_ERR_INVALID;
  if ((uintptr_t)x % dtype_size(dtype) || (uintptr_t)scales % dtype_size(dtype)) return RQ_ERR_ALIGN;
  return int8_quantize_rows(x, dtype, rows, cols, q, scales, (cudaStream_t)stream);
}

int rq_int8_dequantize(const int8_t* q, int64_t numel, const void* scales, int scale_dtype, int block_size,
                       int64_t cols, void* out, int out_dtype, void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(scale_dtype) || !dtype_ok(out_dtype)) return RQ_ERR_DTYPE;
  if (numel < 0 || cols < 0 || (cols == 0 && block_size < 1)) return RQ_ERR_INVALID;
  if (numel == 0) return RQ_OK;
  if (!q || !scales || !out) return RQ_ERR_INVALID;
  if ((uintptr_t)out % dtype_size(out_dtype) || (uintptr_t)scales % dtype_size(scale_dtype)) return RQ_ERR_ALIGN;
  return int8_dequantize(q, numel, scales, scale_dtype, block_size, cols, out, out_dtype, (cudaStream_t)stream);
}

int rq_dq_quantize_scales(const float* c1, int64_t nb, int block2, int fp8, uint8_t* c2, float* c2_scales,
                          void* stream) {
  RQ_PROLOGUE();
  if (nb < 0 || block2 < 1) return RQ_ERR_INVALID;
  if (nb == 0) return RQ_OK;
  if (!c1 || !c2 || !c2_scales) return RQ_ERR_INVALID;
  if ((uintptr_t)c1 % 4 || (uintptr_t)c2_scales % 4) return RQ_ERR_ALIGN;
  return dq_quantize_scales(c1, nb, block2, fp8 ? 1 : 0, c2, c2_scales, (cudaStream_t)stream);
}

int rq_dq_dequantize(const uint8_t* packed, int64_t numel, const uint8_t* c2, const float* c2_scales, int fp8,
                     int block_size, int block2, void* out, int out_dtype, void* stream) {
  RQ_PROLOGUE();
  if (!dtype_ok(out_dtype)) return RQ_ERR_DTYPE;
  if (numel < 0 || block_size < 2 || (block_size & 1) || block2 < 1) return RQ_ERR_INVALID;
  if (numel == 0) return RQ_OK;
  if (!packed || !c2 || !c2_scales || !out) return RQ_ERR_INVALID;
  if ((uintptr_t)out % dtype_size(out_dtype) || (uintptr_t)c2_scales % 4) return RQ_ERR_ALIGN;
  return dq_dequantize(packed, numel, c2, c2_scales, fp8 ? 1 : 0, block_size, block2, out, out_dtype,
                       (cudaStream_t)stream);
}

int64_t rq_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int r) {
  if (M < 0 || N < 0 || K < 0 || r < 0) return -1;
  return linear_workspace_bytes(M, N, K, r);
}

int rq_linear_forward(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                      const float* c2_scales, int64_t N, int64_t K, int block_size, const void* x, int xdtype,
                      int64_t M, const void* lora_x, const void* bias, int bias_dtype, const void* lora_a,
                      const void* lora_b, int r, float scaling, void* y, void* workspace, int64_t workspace_bytes,
                      void* stream) {
  RQ_PROLOGUE();
  LinearArgs a;
  int rc = fill_args(&a, wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size, x, xdtype, M, bias,
                     bias_dtype, lora_a, lora_b, r, scaling, y, workspace, workspace_bytes);
  if (rc != RQ_OK) return rc;
  if (lora_x && (uintptr_t)lora_x % dtype_size(xdtype)) return RQ_ERR_ALIGN;
  a.lora_x = lora_x ? lora_x : x;
  return linear_forward(a, (cudaStream_t)stream);
}

int rq_linear_forward_gather(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                             const float* c2_scales, int64_t N, int64_t K, int block_size, const void* x, int xdtype,
                             int64_t M, const void* bias, int bias_dtype, const void* lora_a, const void* lora_b, int r,
                             float scaling, const RqGather* gather, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  RQ_PROLOGUE();
  if (!gather) return RQ_ERR_INVALID;
  LinearArgs a;
  // the output is the ranks' Y, not a local y: x stands in for the argument
  // check (it is never written)
  int rc = fill_args(&a, wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size, x, xdtype, M, bias,
                     bias_dtype, lora_a, lora_b, r, scaling, const_cast<void*>(x), workspace, workspace_bytes);
  if (rc != RQ_OK) return rc;
  a.y = nullptr;
  a.gather = gather;
  return linear_forward(a, (cudaStream_t)stream);
}

int rq_linear_dx(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                 const float* c2_scales, int64_t N, int64_t K, int block_size, const void* dy, int xdtype, int64_t M,
                 const void* lora_a, const void* lora_b, int r, float scaling, void* dx, void* workspace,
                 int64_t workspace_bytes, void* stream) {
  RQ_PROLOGUE();
  LinearArgs a;
  int rc = fill_args(&a, wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size, dy, xdtype, M,
                     nullptr, 0, lora_a, lora_b, r, scaling, dx, workspace, workspace_bytes);
  if (rc != RQ_OK) return rc;
  return linear_dx(a, (cudaStream_t)stream);
}

int rq_merge_lora(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                  const float* c2_scales, int64_t N, int64_t K, int block_size, const float* lora_a,
                  const float* lora_b, int r, float scaling, int mode, void* out, int out_dtype, void* stream) {
  RQ_PROLOGUE();
  int rc = check_weight(wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size);
  if (rc != RQ_OK) return rc;
  if (!dtype_ok(out_dtype)) return RQ_ERR_DTYPE;
  if (r < 0 || r > 128 || (r > 0 && (!lora_a || !lora_b)) || (N * K > 0 && !out)) return RQ_ERR_INVALID;
  if (mode != RQ_MERGE_FP32_SUM && mode != RQ_MERGE_ROUND_EACH) return RQ_ERR_INVALID;
  if ((uintptr_t)out % dtype_size(out_dtype)) return RQ_ERR_ALIGN;
  const QWeight w{wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size};
  return merge_weight(w, lora_a, lora_b, r, scaling, mode, out, out_dtype, (cudaStream_t)stream);
}

int rq_weight_absmax(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                     const float* c2_scales, int64_t N, int64_t K, int block_size, int dtype, float* absmax,
                     void* stream) {
  RQ_PROLOGUE();
  const int rc = check_weight(wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size);
  if (rc != RQ_OK) return rc;
  if (!dtype_ok(dtype)) return RQ_ERR_DTYPE;
  if (!absmax) return RQ_ERR_INVALID;
  if ((uintptr_t)absmax % 4) return RQ_ERR_ALIGN;
  const QWeight w{wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size};
  return weight_absmax(w, dtype, absmax, (cudaStream_t)stream);
}

int rq_weight_to_fp8(int wfmt, const void* qweight, const void* scales, int scale_dtype, const uint8_t* c2,
                     const float* c2_scales, int64_t N, int64_t K, int block_size, int dtype, float w_scale,
                     uint8_t* fp8_out, void* stream) {
  RQ_PROLOGUE();
  const int rc = check_weight(wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size);
  if (rc != RQ_OK) return rc;
  if (!dtype_ok(dtype)) return RQ_ERR_DTYPE;
  if (N * K > 0 && !fp8_out) return RQ_ERR_INVALID;
  const QWeight w{wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size};
  return weight_to_fp8(w, dtype, w_scale, fp8_out, (cudaStream_t)stream);
}

void launch_int4_dequant_matmul(void* stream, void* x, void* w_packed, void* scales, void* c, int M, int N, int K,
                                int block_size) {
  g_last_status = rq_linear_forward(RQ_W_NF4, w_packed, scales, RQ_F16, nullptr, nullptr, N, K, block_size, x,
                                    RQ_F16, M, nullptr, nullptr, 0, nullptr, nullptr, 0, 1.0f, c, nullptr, 0, stream);
}

void launch_int8_dequant_matmul(void* stream, void* x, void* w_int8, void* scales, void* c, int M, int N, int K,
                                int block_size) {
  g_last_status = rq_linear_forward(RQ_W_INT8, w_int8, scales, RQ_F16, nullptr, nullptr, N, K, block_size, x,
                                    RQ_F16, M, nullptr, nullptr, 0, nullptr, nullptr, 0, 1.0f, c, nullptr, 0, stream);
}

}  // extern "C"
