// merge_kernels.cu -- the merged weight of a LoRA-adapted QuantLinear,
// dequantized and combined with the adapter in one pass over the codes.
//
//   W'[n, k] = deq(W)[n, k] + s * sum_j B[n, j] * A[j, k]
//
// in the two roundings the reference uses:
//   RQ_MERGE_FP32_SUM  (LoRALinear.merge_lora, lora_layer.py:72-113): the
//     fp32 dequantized weight plus the fp32 delta (B @ A, then * s), one
//     rounding to the output dtype;
//   RQ_MERGE_ROUND_EACH (_export_dequant_layer, export/gguf_export.py:30-80):
//     the dequantized weight and the delta each rounded to the output dtype,
//     then added in it.
// The weight codes are read once (HBM-bound: N*K/2 bytes in, 2 bytes out per
// element for fp16); the rank-r delta comes from shared-memory tiles of A
// and B.  A CTA covers 64 rows x 128 columns; a thread 8 consecutive columns
// of 4 rows.
#include <cuda_runtime.h>
#include <string.h>

#include "linear_common.cuh"

namespace rq {

constexpr int kMergeRows = 64, kMergeCols = 128, kMergeThreads = 256;

template <int ODT>
__global__ void __launch_bounds__(kMergeThreads) merge_k(const QWeight w, const float* __restrict__ A,
                                                       const float* __restrict__ B, int r, float s, int mode,
                                                       typename DType<ODT>::T* __restrict__ out) {
  using T = typename DType<ODT>::T;
  extern __shared__ __align__(16) float msm[];
  float* a_t = msm;                           // [r][kMergeCols]
  float* b_t = msm + r * kMergeCols;          // [kMergeRows][r]
  __shared__ float lut16[16];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t K = w.K, N = w.N;
  const int64_t c0 = (int64_t)blockIdx.x * kMergeCols, r0 = (int64_t)blockIdx.y * kMergeRows;
  if (tid < 16) lut16[tid] = kNF4[tid];
  for (int i = tid; i < r * kMergeCols; i += kMergeThreads) {
    const int j = i / kMergeCols, c = i - j * kMergeCols;
    a_t[i] = (c0 + c < K) ? A[(int64_t)j * K + c0 + c] : 0.0f;
  }
  for (int i = tid; i < kMergeRows * r; i += kMergeThreads) {
    const int rr = i / r, j = i - rr * r;
    b_t[i] = (r0 + rr < N) ? B[(r0 + rr) * r + j] : 0.0f;
  }
  __syncthreads();
  const int64_t k0 = c0 + tx * 8;
#pragma unroll 1
  for (int i = 0; i < kMergeRows / 16; ++i) {
    const int rr = ty + 16 * i;
    const int64_t n = r0 + rr;
    if (n >= N) break;
    float d[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) d[e] = 0.0f;
    for (int j = 0; j < r; ++j) {  // in order of j, as one dot product per element
      const float bv = b_t[rr * r + j];
      const float4 a0 = *reinterpret_cast<const float4*>(a_t + j * kMergeCols + tx * 8);
      const float4 a1 = *reinterpret_cast<const float4*>(a_t + j * kMergeCols + tx * 8 + 4);
      d[0] = fmaf(bv, a0.x, d[0]), d[1] = fmaf(bv, a0.y, d[1]), d[2] = fmaf(bv, a0.z, d[2]);
      d[3] = fmaf(bv, a0.w, d[3]), d[4] = fmaf(bv, a1.x, d[4]), d[5] = fmaf(bv, a1.y, d[5]);
      d[6] = fmaf(bv, a1.z, d[6]), d[7] = fmaf(bv, a1.w, d[7]);
    }
    T v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k >= K) {
        v[e] = DType<ODT>::from_f32(0.0f);
        continue;
      }
      const float wv = deq_elem(w, n * K + k, lut16);
      const float delta = d[e] * s;  // (B @ A) * scaling: the product, then the scale
      v[e] = mode == RQ_MERGE_FP32_SUM
                 ? DType<ODT>::from_f32(wv + delta)
                 : DType<ODT>::from_f32(round_to<ODT>(wv) + round_to<ODT>(delta));
    }
    T* orow = out + n * K + k0;
    if (sizeof(T) == 2 && k0 + 8 <= K && ((uintptr_t)orow % 16) == 0) {
      uint4 pk;
      memcpy(&pk, v, sizeof(pk));
      *reinterpret_cast<uint4*>(orow) = pk;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (k0 + e < K) orow[e] = v[e];
    }
  }
}

template <int ODT>
static int merge_launch(const QWeight& w, const float* A, const float* B, int r, float s, int mode, void* out,
                        cudaStream_t st) {
  const size_t smem = (size_t)r * (kMergeCols + kMergeRows) * sizeof(float);
  const int rc = ensure_smem_limit((const void*)merge_k<ODT>, smem);
  if (rc != RQ_OK) return rc;
  const dim3 grid((unsigned)((w.K + kMergeCols - 1) / kMergeCols), (unsigned)((w.N + kMergeRows - 1) / kMergeRows));
  merge_k<ODT><<<grid, kMergeThreads, smem, st>>>(w, A, B, r, s, mode, static_cast<typename DType<ODT>::T*>(out));
  return check_launch();
}

int merge_weight(const QWeight& w, const float* A, const float* B, int r, float s, int mode, void* out, int odt,
                 cudaStream_t st) {
  if (w.N == 0 || w.K == 0) return RQ_OK;
  if ((w.N + kMergeRows - 1) / kMergeRows > 65535) return RQ_ERR_INVALID;
  switch (odt) {
    case RQ_F16: return merge_launch<RQ_F16>(w, A, B, r, s, mode, out, st);
    case RQ_BF16: return merge_launch<RQ_BF16>(w, A, B, r, s, mode, out, st);
    case RQ_F32: return merge_launch<RQ_F32>(w, A, B, r, s, mode, out, st);
  }
  return RQ_ERR_DTYPE;
}

}  // namespace rq
