// noalloc.cu -- rq_linear_forward_noalloc: the QuantLinear+LoRA forward for
// callers that cannot allocate device memory.
//
// Some callers have no way to provide the workspace rq_linear_forward
// needs: plugin hosts that own all device memory through their own
// allocator and hand none out, language bindings (cgo, JNI, plain FFI) that
// have no CUDA allocator of their own, and latency-critical loops where a
// cudaMalloc/cudaFree would synchronize the device.  This entry point runs
// the same forward computation with its scratch taken from a fixed array
// compiled into the library, so it allocates nothing.
//
// The array lives in device global memory of every GPU that loads the
// library, kNoAllocScratchBytes each, until the process exits.  Host code
// cannot use the array's name as a device address (it names a host-side
// stand-in); its device address is looked up with cudaGetSymbolAddress the
// first time the entry point runs on a device, with that device current, and
// again after the device's context was replaced (cudaDeviceReset).  That
// first call should therefore be made before any stream capture.
//
// All calls on a device share the one array and it keeps whatever the last
// call left there; the part that must start at zero (the arrival counters)
// is cleared on the caller's stream at every call.  Calls that may overlap
// on the GPU (different streams, or different host threads without
// ordering) race on the array and must not be issued.
#include <cuda_runtime.h>

#include <mutex>

#include "rq_internal.h"

namespace rq {

constexpr size_t kNoAllocScratchBytes = RQ_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch must keep 256-byte alignment");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Unique id of the calling thread's current CUDA context (cuCtxGetId, never
// reused within a process), through the runtime's driver entry points so
// the library does not link libcuda itself.  0 if the driver cannot say.
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);
static unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != 0 || ctx == nullptr || get_id(ctx, &id) != 0) return 0;
  return id;
}

// Device address of g_noalloc_scratch for the current device and context.
// The address is looked up with cudaGetSymbolAddress the first time a
// device is used and again whenever the device's context has changed (after
// cudaDeviceReset the module is loaded anew and the old address is gone).
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  static unsigned long long ctx_of[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return RQ_ERR_DEVICE;
  // 0 before the thread has a context (the lookup below creates it) or when
  // the driver cannot tell: then the address is looked up again
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr || ctx == 0 || ctx != ctx_of[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_cuda_error(e);
      return RQ_ERR_CUDA;
    }
    addr[dev] = p;
    ctx_of[dev] = current_context_id();
  }
  *out = addr[dev];
  return RQ_OK;
}

}  // namespace rq

extern "C" int rq_linear_forward_noalloc(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                                         const uint8_t* c2, const float* c2_scales, int64_t N, int64_t K,
                                         int block_size, const void* x, int xdtype, int64_t M, const void* lora_x,
                                         const void* bias, int bias_dtype, const void* lora_a, const void* lora_b,
                                         int r, float scaling, void* y, void* stream) {
  if (M < 0 || N < 0 || K < 0 || r < 0) return RQ_ERR_INVALID;
  const int64_t need = rq_linear_workspace_bytes(M, N, K, r);
  if (need < 0) return RQ_ERR_INVALID;
  if ((uint64_t)need > rq::kNoAllocScratchBytes) return RQ_ERR_SCRATCH;
  void* scratch = nullptr;
  int rc = rq::noalloc_scratch(&scratch);
  if (rc != RQ_OK) return rc;
  // the counter area must be zero when a call starts
  cudaError_t e = cudaMemsetAsync(scratch, 0, 256, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    rq::set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return rq_linear_forward(wfmt, qweight, scales, scale_dtype, c2, c2_scales, N, K, block_size, x, xdtype, M,
                           lora_x, bias, bias_dtype, lora_a, lora_b, r, scaling, y, scratch,
                           (int64_t)rq::kNoAllocScratchBytes, stream);
}
