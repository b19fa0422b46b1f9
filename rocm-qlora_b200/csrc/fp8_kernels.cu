// fp8_kernels.cu -- the quantized weight of a QuantLinear as a per-tensor
// scaled float8_e4m3fn operand for an FP8 GEMM (FP8LinearWrapper's native
// path, rocm_qlora/fp8/fp8_linear.py:27-39 of the reference):
//
//   w      = rnd_DT(deq(W))                 the weight .to(x.dtype)
//   amax   = max |w|                        rq_weight_absmax
//   s      = amax / 448 (fp32)              the caller
//   w_f8   = e4m3fn(rnd_DT(w / rnd_DT(s)))  rq_weight_to_fp8: torch's GPU
//                                           division of a DT tensor by a 0-dim
//                                           fp32 device tensor converts the
//                                           divisor to DT first, then divides
//                                           in fp32 and rounds to DT; then RNE
//                                           to e4m3fn (no saturation)
//
// Both kernels read the codes straight from the quantized buffers (no bf16
// copy of the weight is made); they run once per weight version, since the
// base weight of a QLoRA layer is frozen.  Each thread takes 16 consecutive
// flat elements; |w| >= 0, so the fp32 bit patterns order like the values
// and the maximum is an integer atomicMax.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "linear_common.cuh"

namespace rq {

constexpr int kFp8Threads = 256, kFp8Per = 16;

template <int DT>
__global__ void __launch_bounds__(kFp8Threads) weight_absmax_k(const QWeight w, unsigned* __restrict__ out_bits) {
  __shared__ float lut16[16];
  if (threadIdx.x < 16) lut16[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int64_t n = w.N * w.K;
  float m = 0.0f;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c * kFp8Per < n;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = c * kFp8Per;
#pragma unroll 4
    for (int i = 0; i < kFp8Per; ++i)
      if (e0 + i < n) m = fmaxf(m, fabsf(round_to<DT>(deq_elem(w, e0 + i, lut16))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));
}

template <int DT>
__global__ void __launch_bounds__(kFp8Threads) weight_to_fp8_k(const QWeight w, float s,
                                                               uint8_t* __restrict__ out) {
  __shared__ float lut16[16];
  if (threadIdx.x < 16) lut16[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int64_t n = w.N * w.K;
  const float sd = round_to<DT>(s);
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c * kFp8Per < n;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = c * kFp8Per;
    uint8_t v[kFp8Per];
#pragma unroll
    for (int i = 0; i < kFp8Per; ++i) {
      const float wv = e0 + i < n ? round_to<DT>(deq_elem(w, e0 + i, lut16)) : 0.0f;
      v[i] = (uint8_t)__nv_cvt_float_to_fp8(round_to<DT>(ieee_div(wv, sd)), __NV_NOSAT, __NV_E4M3);
    }
    if (e0 + kFp8Per <= n && ((uintptr_t)(out + e0) % 16) == 0) {
      uint4 pk;
      memcpy(&pk, v, sizeof(pk));
      *reinterpret_cast<uint4*>(out + e0) = pk;
    } else {
      for (int i = 0; i < kFp8Per && e0 + i < n; ++i) out[e0 + i] = v[i];
    }
  }
}

static int fp8_grid(int64_t n) {
  const int64_t chunks = (n + kFp8Per - 1) / kFp8Per;
  int64_t g = (chunks + kFp8Threads - 1) / kFp8Threads;
  return (int)(g < 1 ? 1 : (g > 148 * 16 ? 148 * 16 : g));
}

int weight_absmax(const QWeight& w, int dt, float* out, cudaStream_t st) {
  unsigned* bits = reinterpret_cast<unsigned*>(out);
  cudaError_t e = cudaMemsetAsync(bits, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  if (w.N * w.K == 0) return RQ_OK;
  const int g = fp8_grid(w.N * w.K);
  switch (dt) {
    case RQ_BF16: weight_absmax_k<RQ_BF16><<<g, kFp8Threads, 0, st>>>(w, bits); break;
    case RQ_F16: weight_absmax_k<RQ_F16><<<g, kFp8Threads, 0, st>>>(w, bits); break;
    case RQ_F32: weight_absmax_k<RQ_F32><<<g, kFp8Threads, 0, st>>>(w, bits); break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

int weight_to_fp8(const QWeight& w, int dt, float s, uint8_t* out, cudaStream_t st) {
  if (w.N * w.K == 0) return RQ_OK;
  const int g = fp8_grid(w.N * w.K);
  switch (dt) {
    case RQ_BF16: weight_to_fp8_k<RQ_BF16><<<g, kFp8Threads, 0, st>>>(w, s, out); break;
    case RQ_F16: weight_to_fp8_k<RQ_F16><<<g, kFp8Threads, 0, st>>>(w, s, out); break;
    case RQ_F32: weight_to_fp8_k<RQ_F32><<<g, kFp8Threads, 0, st>>>(w, s, out); break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

}  // namespace rq
