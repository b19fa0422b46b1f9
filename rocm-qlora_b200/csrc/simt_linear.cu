// simt_linear.cu -- exact per-element QuantLinear+LoRA kernels on CUDA cores.
//
// This is the literal restatement of the reference's eager path
// (quant_linear.py:182-197 + lora_layer.py:63-70): every weight element is
// dequantized in fp32 exactly as dequantize_* does, rounded to the
// activation dtype (`weight_fp.to(x.dtype)`), and multiplied with fp32
// accumulation.  It serves fp32 activations (config 1 of the benchmark is
// fp32) and shapes the tensor-core kernels do not take (K not a multiple of
// 64, blocks that straddle rows, odd block sizes); it is not a fallback for
// the tensor-core paths -- the dispatcher picks exactly one kernel per shape.
#include <cuda_runtime.h>

#include "linear_common.cuh"

namespace rq {

constexpr int kSimtTN = 64;  // outputs along N (or K for dx) per CTA
constexpr int kSimtTM = 8;   // rows of M per CTA (2 per thread)

// y[m, n] = epilogue(sum_k x[m,k] * rnd(deq(W[n,k])))
template <int DT>
__global__ void __launch_bounds__(256) simt_forward_k(QWeight w, const typename DType<DT>::T* __restrict__ x,
                                                      int64_t M, const void* bias, int bdt,
                                                      const typename DType<DT>::T* __restrict__ tdown,
                                                      const typename DType<DT>::T* __restrict__ lora_b, int r,
                                                      float s, typename DType<DT>::T* __restrict__ y) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int64_t N = w.N, K = w.K;
  const int64_t n = (int64_t)blockIdx.x * kSimtTN + (threadIdx.x % kSimtTN);
  const int64_t m0 = (int64_t)blockIdx.y * kSimtTM + (threadIdx.x / kSimtTN) * 2;
  if (n >= N) return;
  float acc0 = 0.0f, acc1 = 0.0f;
  const bool has1 = m0 + 1 < M;
  if (m0 < M) {
    const auto* x0 = x + m0 * K;
    const auto* x1 = x + (has1 ? m0 + 1 : m0) * K;
    for (int64_t k = 0; k < K; ++k) {
      const float wv = round_to<DT>(deq_elem(w, n * K + k, lut));
      acc0 = fmaf(DType<DT>::to_f32(x0[k]), wv, acc0);
      acc1 = fmaf(DType<DT>::to_f32(x1[k]), wv, acc1);
    }
  }
  const bool has_bias = bias != nullptr;
  const float bv = has_bias ? load_scalar(bias, bdt, n) : 0.0f;
  const bool has_lora = r > 0;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int64_t m = m0 + e;
    if (m >= M) break;
    float u = 0.0f;
    for (int j = 0; j < r; ++j)
      u = fmaf(DType<DT>::to_f32(tdown[m * r + j]), DType<DT>::to_f32(lora_b[n * r + j]), u);
    y[m * N + n] = DType<DT>::from_f32(lora_epilogue<DT>(e ? acc1 : acc0, has_bias, bv, u, has_lora, s));
  }
}

// dx[m, k] = rnd(rnd(sum_n dy[m,n] * rnd(deq(W[n,k]))) + rnd(sum_j gt[m,j] A[j,k]))
template <int DT>
__global__ void __launch_bounds__(256) simt_dx_k(QWeight w, const typename DType<DT>::T* __restrict__ dy, int64_t M,
                                                 const typename DType<DT>::T* __restrict__ gt,
                                                 const typename DType<DT>::T* __restrict__ lora_a, int r,
                                                 typename DType<DT>::T* __restrict__ dx) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int64_t N = w.N, K = w.K;
  const int64_t k = (int64_t)blockIdx.x * kSimtTN + (threadIdx.x % kSimtTN);
  const int64_t m0 = (int64_t)blockIdx.y * kSimtTM + (threadIdx.x / kSimtTN) * 2;
  if (k >= K) return;
  float acc0 = 0.0f, acc1 = 0.0f;
  const bool has1 = m0 + 1 < M;
  if (m0 < M) {
    const auto* d0 = dy + m0 * N;
    const auto* d1 = dy + (has1 ? m0 + 1 : m0) * N;
    for (int64_t n = 0; n < N; ++n) {
      const float wv = round_to<DT>(deq_elem(w, n * K + k, lut));
      acc0 = fmaf(DType<DT>::to_f32(d0[n]), wv, acc0);
      acc1 = fmaf(DType<DT>::to_f32(d1[n]), wv, acc1);
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int64_t m = m0 + e;
    if (m >= M) break;
    float u = 0.0f;
    for (int j = 0; j < r; ++j)
      u = fmaf(DType<DT>::to_f32(gt[m * r + j]), DType<DT>::to_f32(lora_a[(int64_t)j * K + k]), u);
    dx[m * K + k] = DType<DT>::from_f32(lora_epilogue<DT>(e ? acc1 : acc0, false, 0.0f, u, r > 0, 1.0f));
  }
}

template <int DT>
static int simt_fwd_t(const LinearArgs& a, const void* tdown, cudaStream_t st) {
  using T = typename DType<DT>::T;
  const dim3 grid((unsigned)((a.w.N + kSimtTN - 1) / kSimtTN), (unsigned)((a.M + kSimtTM - 1) / kSimtTM));
  if (grid.y > 65535) return RQ_ERR_INVALID;
  simt_forward_k<DT><<<grid, 256, 0, st>>>(a.w, (const T*)a.x, a.M, a.bias, a.bdt, (const T*)tdown,
                                           (const T*)a.lora_b, a.r, a.scaling, (T*)a.y);
  return check_launch();
}

template <int DT>
static int simt_dx_t(const LinearArgs& a, const void* gt, cudaStream_t st) {
  using T = typename DType<DT>::T;
  const dim3 grid((unsigned)((a.w.K + kSimtTN - 1) / kSimtTN), (unsigned)((a.M + kSimtTM - 1) / kSimtTM));
  if (grid.y > 65535) return RQ_ERR_INVALID;
  simt_dx_k<DT><<<grid, 256, 0, st>>>(a.w, (const T*)a.x, a.M, (const T*)gt, (const T*)a.lora_a, a.r, (T*)a.y);
  return check_launch();
}

int simt_forward(const LinearArgs& a, const void* tdown, cudaStream_t st) {
  switch (a.xdt) {
    case RQ_F32: return simt_fwd_t<RQ_F32>(a, tdown, st);
    case RQ_BF16: return simt_fwd_t<RQ_BF16>(a, tdown, st);
    case RQ_F16: return simt_fwd_t<RQ_F16>(a, tdown, st);
  }
  return RQ_ERR_DTYPE;
}

int simt_dx(const LinearArgs& a, const void* gt, cudaStream_t st) {
  switch (a.xdt) {
    case RQ_F32: return simt_dx_t<RQ_F32>(a, gt, st);
    case RQ_BF16: return simt_dx_t<RQ_BF16>(a, gt, st);
    case RQ_F16: return simt_dx_t<RQ_F16>(a, gt, st);
  }
  return RQ_ERR_DTYPE;
}

}  // namespace rq
