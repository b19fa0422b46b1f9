// quant_kernels.cu -- NF4 / INT8 / double-quant quantize and dequantize.
//
// These are HBM streaming kernels over the flat weight tensor, the layout of
// rocm_qlora/quantization/quant_ops.py (blocks of `bs` consecutive flat
// elements, zero padded at the end).  Each thread moves 16 bytes per access
// (float4 / 8 x bf16); the absmax of a block is a shuffle reduction over the
// lanes that hold it.  The arithmetic per element follows the reference's
// torch ops exactly (see rq_common.cuh), so codes and scales are bit-exact.
#include <cuda_runtime.h>

#include "rq_common.cuh"
#include "rq_internal.h"

namespace rq {

// ---------------------------------------------------------------- NF4 quant
//
// For bf16 / f16 inputs the normalized value x / absmax is a 16-bit value in
// [-1, 1] (|x| <= absmax, absmax >= 1e-12 after the clamp), or NaN.  Its code
// nf4_code(value) then depends only on the 16-bit pattern: every |value| <
// 2^-5 lies between the thresholds of code 7, and the patterns from 2^-5 to
// 1 are few (641 bf16, 5121 f16 a sign).  A per-CTA table holds
//   entry 0                 code 7 (|value| < 2^-5)
//   entry 1 + (a - lo)      nf4_code of pattern a, lo <= a <= 1.0
//   entry 2 + (1.0 - lo)    code 0 (NaN; +inf cannot occur)
// for each sign, built with nf4_code itself, so a lookup equals nf4_code
// for every value the kernel can meet.
template <int DT> struct QTab;
template <> struct QTab<RQ_BF16> {
  static constexpr uint32_t kLo = 0x3D00u, kOne = 0x3F80u, kSign = 0x400u, kSize = 2 * kSign;
  static __device__ __forceinline__ uint32_t bits(float q) { return __bfloat16_as_ushort(__float2bfloat16_rn(q)); }
  static __device__ __forceinline__ float value(uint32_t b) { return __uint_as_float(b << 16); }
  static __device__ __forceinline__ uint32_t sign(uint32_t b) { return (b >> 5) & kSign; }
};
template <> struct QTab<RQ_F16> {
  static constexpr uint32_t kLo = 0x2800u, kOne = 0x3C00u, kSign = 0x2000u, kSize = 2 * kSign;
  static __device__ __forceinline__ uint32_t bits(float q) { return __half_as_ushort(__float2half_rn(q)); }
  static __device__ __forceinline__ float value(uint32_t b) {
    return __half2float(__ushort_as_half((unsigned short)b));
  }
  static __device__ __forceinline__ uint32_t sign(uint32_t b) { return (b >> 2) & kSign; }
};
template <> struct QTab<RQ_F32> {  // fp32 inputs keep the threshold search
  static constexpr uint32_t kSize = 4;
};

template <int DT>
__device__ __forceinline__ void qtab_build(uint8_t* tab) {
  using Q = QTab<DT>;
  for (uint32_t e = threadIdx.x; e < Q::kSize; e += blockDim.x) {
    const uint32_t j = e & (Q::kSign - 1), neg = e & Q::kSign;
    int c = 0;
    if (j == 0) {
      c = 7;
    } else if (j <= Q::kOne - Q::kLo + 1) {
      const uint32_t a = Q::kLo + j - 1;
      c = nf4_code(Q::value(neg ? (a | 0x8000u) : a));
    }
    tab[e] = (uint8_t)c;
  }
}

// code of x / scale (the reference's x_norm, rounded to DT) from the table
template <int DT>
__device__ __forceinline__ int qtab_code(float q, const uint8_t* tab) {
  using Q = QTab<DT>;
  const uint32_t b = Q::bits(q), a = b & 0x7FFFu;
  int j = (int)a - (int)(Q::kLo - 1);
  j = j < 0 ? 0 : j;
  j = j > (int)(Q::kOne - Q::kLo + 2) ? (int)(Q::kOne - Q::kLo + 2) : j;
  return tab[(uint32_t)j | Q::sign(b)];
}

// Fast path: VEC = 16/sizeof(T) elements per lane, L = bs/VEC lanes per
// block (L in {1,...,32}).  Each warp covers 32*VEC elements = 32/L blocks.
template <int DT, int L>
__global__ void __launch_bounds__(256) nf4_quantize_vec(const typename DType<DT>::T* __restrict__ x,
                                                        int64_t n, int64_t nb, uint8_t* __restrict__ packed,
                                                        typename DType<DT>::T* __restrict__ scales) {
  using T = typename DType<DT>::T;
  constexpr int VEC = 16 / sizeof(T);
  constexpr int BS = VEC * L;
  __shared__ uint8_t qtab[QTab<DT>::kSize];
  if constexpr (DT != RQ_F32) {
    qtab_build<DT>(qtab);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t blocks_per_warp = 32 / L;
  for (int64_t wb = warp * blocks_per_warp; wb < nb; wb += nwarps * blocks_per_warp) {
    const int64_t blk = wb + lane / L;
    const int64_t e0 = blk * BS + (int64_t)(lane % L) * VEC;
    float v[VEC];
    if (blk < nb && e0 + VEC <= n) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + e0);
      const T* t = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < VEC; ++i) v[i] = DType<DT>::to_f32(t[i]);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) v[i] = (blk < nb && e0 + i < n) ? DType<DT>::to_f32(x[e0 + i]) : 0.0f;
    }
    float amax = 0.0f;
    bool nan = false;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      nan |= isnan(v[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = seg_max<L>(amax);
    nan = seg_any<L>(nan);
    const float scale = nan ? __uint_as_float(0x7fc00000u) : clamp_eps<DT>(amax);
    if (blk < nb) {
      if (lane % L == 0) scales[blk] = DType<DT>::from_f32(scale);
      uint32_t bytes[VEC / 8 > 0 ? VEC / 8 : 1] = {0};
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        int c;
        if constexpr (DT == RQ_F32) c = nf4_code(ieee_div(v[i], scale));
        else c = qtab_code<DT>(ieee_div(v[i], scale), qtab);
        bytes[i / 8] |= (uint32_t)c << (4 * (i % 8));
      }
      if constexpr (VEC == 4) {
        *reinterpret_cast<uint16_t*>(packed + e0 / 2) = (uint16_t)bytes[0];
      } else {
        *reinterpret_cast<uint32_t*>(packed + e0 / 2) = bytes[0];
      }
    }
  }
}

// Generic path: one warp per block, any even block size.
template <int DT>
__global__ void __launch_bounds__(256) nf4_quantize_generic(const typename DType<DT>::T* __restrict__ x,
                                                            int64_t n, int64_t nb, int bs,
                                                            uint8_t* __restrict__ packed,
                                                            typename DType<DT>::T* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < nb; b += nwarps) {
    const int64_t base = b * bs;
    float amax = 0.0f;
    bool nan = false;
    for (int j = lane; j < bs; j += 32) {
      const int64_t i = base + j;
      const float v = i < n ? DType<DT>::to_f32(x[i]) : 0.0f;
      nan |= isnan(v);
      amax = fmaxf(amax, fabsf(v));
    }
    amax = seg_max<32>(amax);
    nan = __any_sync(0xffffffffu, nan);
    const float scale = nan ? __uint_as_float(0x7fc00000u) : clamp_eps<DT>(amax);
    if (lane == 0) scales[b] = DType<DT>::from_f32(scale);
    for (int j = 2 * lane; j < bs; j += 64) {
      int c[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t i = base + j + e;
        const float v = i < n ? DType<DT>::to_f32(x[i]) : 0.0f;
        c[e] = nf4_code(round_to<DT>(ieee_div(v, scale)));
      }
      packed[(base + j) / 2] = (uint8_t)(c[0] | (c[1] << 4));
    }
  }
}

template <int DT>
static int launch_nf4_quantize(const void* x, int64_t n, int bs, uint8_t* packed, void* scales,
                               cudaStream_t st) {
  using T = typename DType<DT>::T;
  constexpr int VEC = 16 / sizeof(T);
  const int64_t nb = (n + bs - 1) / bs;
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((uintptr_t)packed % 4 == 0);
  const int threads = 256;
  auto grid_for = [&](int64_t warps_needed) {
    int64_t g = (warps_needed * 32 + threads - 1) / threads;
    // a persistent grid (8 CTAs an SM): each CTA builds its code table once
    return (int)(g < 148 * 8 ? (g < 1 ? 1 : g) : 148 * 8);
  };
  const T* xp = static_cast<const T*>(x);
  T* sp = static_cast<T*>(scales);
  if (aligned && bs % VEC == 0) {
    const int L = bs / VEC;
    const int64_t warps = (nb * L + 31) / 32;
    switch (L) {
#define RQ_CASE(LL)                                                                          \
  case LL:                                                                                   \
    nf4_quantize_vec<DT, LL><<<grid_for(warps), threads, 0, st>>>(xp, n, nb, packed, sp); \
    return check_launch();
      RQ_CASE(1) RQ_CASE(2) RQ_CASE(4) RQ_CASE(8) RQ_CASE(16) RQ_CASE(32)
#undef RQ_CASE
      default: break;
    }
  }
  nf4_quantize_generic<DT><<<grid_for(nb), threads, 0, st>>>(xp, n, nb, bs, packed, sp);
  return check_launch();
}

// -------------------------------------------------------------- NF4 dequant
// Each thread expands 8 packed bytes (16 values).  Blocks of >= 16 elements
// that are multiples of 16 keep one scale per thread chunk.  The block scale
// comes from a scale source: the plain per-block scales, or (double quant)
// the second-level code times its group's c2_scales entry.
template <int SDT>
struct PlainScales {
  const typename DType<SDT>::T* s;
  __device__ __forceinline__ float operator()(int64_t b) const { return DType<SDT>::to_f32(s[b]); }
};
// double_dequantize (double_quant.py:99-122): c1 = decode(c2) * c2_scales
struct DqScales {
  const uint8_t* c2;
  const float* c2s;
  int fp8, bs2;
  __device__ __forceinline__ float operator()(int64_t b) const {
    const float q = fp8 ? e4m3fnuz_to_f32(c2[b]) : ieee_div((float)(int8_t)c2[b], 127.0f);
    return q * c2s[b / bs2];
  }
};

template <class SF, int ODT>
__global__ void __launch_bounds__(256) nf4_dequantize_k(const uint8_t* __restrict__ packed, int64_t nv,
                                                        const SF sf, int bs,
                                                        typename DType<ODT>::T* __restrict__ out) {
  // nv values (packed holds ceil(nv / 2) bytes)
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int64_t nchunks = (nv + 15) / 16;
  const bool fast_scale = (bs % 16) == 0;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b0 = c * 8;
    const int64_t e0 = b0 * 2;
    if (e0 + 16 <= nv && ((uintptr_t)(packed + b0) % 8 == 0)) {
      const uint2 raw = *reinterpret_cast<const uint2*>(packed + b0);
      const uint32_t w[2] = {raw.x, raw.y};
      const float s = fast_scale ? sf(e0 / bs) : 0.0f;
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int code = (w[i / 8] >> (4 * (i % 8))) & 0xF;
        const float si = fast_scale ? s : sf((e0 + i) / bs);
        v[i] = lut[code] * si;
      }
      if constexpr (ODT == RQ_F32) {
        float4* o = reinterpret_cast<float4*>(out + e0);
        if (((uintptr_t)o % 16) == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) out[e0 + i] = v[i];
        }
      } else {
        if (((uintptr_t)(out + e0) % 16) == 0) {
          uint32_t h[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) h[i] = pack2<ODT>(v[2 * i], v[2 * i + 1]);
          uint4* o = reinterpret_cast<uint4*>(out + e0);
          o[0] = make_uint4(h[0], h[1], h[2], h[3]);
          o[1] = make_uint4(h[4], h[5], h[6], h[7]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) out[e0 + i] = DType<ODT>::from_f32(v[i]);
        }
      }
    } else {
      for (int64_t i = e0; i < nv && i < e0 + 16; ++i) {
        const uint8_t byte = packed[i >> 1];
        const int code = (i & 1) ? (byte >> 4) : (byte & 0xF);
        out[i] = DType<ODT>::from_f32(lut[code] * sf(i / bs));
      }
    }
  }
}

// ------------------------------------------------------- DQ second level
// One warp per group of bs2 first-level scales.
__global__ void __launch_bounds__(256) dq_quantize_scales_k(const float* __restrict__ c1, int64_t nb, int bs2,
                                                            int fp8, uint8_t* __restrict__ c2,
                                                            float* __restrict__ c2s) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t ng = (nb + bs2 - 1) / bs2;
  for (int64_t g = warp; g < ng; g += nwarps) {
    float amax = 0.0f;
    bool nan = false;
    for (int j = lane; j < bs2; j += 32) {
      const int64_t i = g * bs2 + j;
      const float v = i < nb ? c1[i] : 0.0f;
      nan |= isnan(v);
      amax = fmaxf(amax, fabsf(v));
    }
    amax = seg_max<32>(amax);
    nan = __any_sync(0xffffffffu, nan);
    const float s = nan ? __uint_as_float(0x7fc00000u) : clamp_eps<RQ_F32>(amax);
    if (lane == 0) c2s[g] = s;
    for (int j = lane; j < bs2; j += 32) {
      const int64_t i = g * bs2 + j;
      const float v = i < nb ? c1[i] : 0.0f;
      const float nrm = ieee_div(v, s);
      c2[i] = fp8 ? f32_to_e4m3fnuz(nrm) : (uint8_t)to_int8_torch(rintf(nrm * 127.0f));
    }
  }
}

// ---------------------------------------------------------------- INT8
template <int DT>
__global__ void __launch_bounds__(256) int8_quantize_k(const typename DType<DT>::T* __restrict__ x, int64_t n,
                                                       int64_t nb, int bs, int8_t* __restrict__ q,
                                                       typename DType<DT>::T* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp; b < nb; b += nwarps) {
    const int64_t base = b * bs;
    float amax = 0.0f;
    bool nan = false;
    for (int j = lane; j < bs; j += 32) {
      const int64_t i = base + j;
      const float v = i < n ? DType<DT>::to_f32(x[i]) : 0.0f;
      nan |= isnan(v);
      amax = fmaxf(amax, fabsf(v));
    }
    amax = seg_max<32>(amax);
    nan = __any_sync(0xffffffffu, nan);
    float s = nan ? __uint_as_float(0x7fc00000u) : round_to<DT>(ieee_div(amax, 127.0f));
    s = clamp_eps<DT>(s);
    if (lane == 0) scales[b] = DType<DT>::from_f32(s);
    for (int j = lane; j < bs; j += 32) {
      const int64_t i = base + j;
      const float v = i < n ? DType<DT>::to_f32(x[i]) : 0.0f;
      q[i] = to_int8_torch(round_to<DT>(rintf(round_to<DT>(ieee_div(v, s)))));
    }
  }
}

// One CTA per row.
template <int DT>
__global__ void __launch_bounds__(256) int8_quantize_rows_k(const typename DType<DT>::T* __restrict__ x,
                                                            int64_t cols, int8_t* __restrict__ q,
                                                            typename DType<DT>::T* __restrict__ scales) {
  __shared__ float red[8];
  __shared__ int rnan[8];
  const int64_t row = blockIdx.x;
  const auto* xr = x + row * cols;
  float amax = 0.0f;
  bool nan = false;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = DType<DT>::to_f32(xr[c]);
    nan |= isnan(v);
    amax = fmaxf(amax, fabsf(v));
  }
  amax = seg_max<32>(amax);
  nan = __any_sync(0xffffffffu, nan);
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = amax;
    rnan[threadIdx.x >> 5] = nan;
  }
  __syncthreads();
  float m = 0.0f;
  bool anynan = false;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    m = fmaxf(m, red[w]);
    anynan |= rnan[w] != 0;
  }
  float s = anynan ? __uint_as_float(0x7fc00000u) : round_to<DT>(ieee_div(m, 127.0f));
  s = clamp_eps<DT>(s);
  if (threadIdx.x == 0) scales[row] = DType<DT>::from_f32(s);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = DType<DT>::to_f32(xr[c]);
    q[row * cols + c] = to_int8_torch(round_to<DT>(rintf(round_to<DT>(ieee_div(v, s)))));
  }
}

template <int SDT, int ODT>
__global__ void __launch_bounds__(256) int8_dequantize_k(const int8_t* __restrict__ q, int64_t n,
                                                         const typename DType<SDT>::T* __restrict__ scales,
                                                         int bs, int64_t cols,
                                                         typename DType<ODT>::T* __restrict__ out) {
  // 16 values a thread: one 16-byte load, one scale when the scale
  // period (cols, or bs) is a multiple of 16
  const int64_t per = cols > 0 ? cols : (int64_t)bs;
  const bool one_scale = per % 16 == 0;
  const int64_t nchunks = (n + 15) / 16;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = c * 16;
    if (one_scale && e0 + 16 <= n && ((uintptr_t)(q + e0) % 16) == 0 && ((uintptr_t)(out + e0) % 16) == 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(q + e0);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      const float s = DType<SDT>::to_f32(scales[e0 / per]);
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = (float)(int8_t)(w[i / 4] >> (8 * (i % 4))) * s;
      if constexpr (ODT == RQ_F32) {
        float4* o = reinterpret_cast<float4*>(out + e0);
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      } else {
        uint32_t h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = pack2<ODT>(v[2 * i], v[2 * i + 1]);
        uint4* o = reinterpret_cast<uint4*>(out + e0);
        o[0] = make_uint4(h[0], h[1], h[2], h[3]);
        o[1] = make_uint4(h[4], h[5], h[6], h[7]);
      }
    } else {
      for (int64_t i = e0; i < n && i < e0 + 16; ++i)
        out[i] = DType<ODT>::from_f32((float)q[i] * DType<SDT>::to_f32(scales[i / per]));
    }
  }
}

static int grid_1d(int64_t work, int threads = 256) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

// ------------------------------------------------------------ dispatchers

int nf4_quantize(const void* x, int dtype, int64_t n, int bs, uint8_t* packed, void* scales, cudaStream_t st) {
  switch (dtype) {
    case RQ_F32: return launch_nf4_quantize<RQ_F32>(x, n, bs, packed, scales, st);
    case RQ_BF16: return launch_nf4_quantize<RQ_BF16>(x, n, bs, packed, scales, st);
    case RQ_F16: return launch_nf4_quantize<RQ_F16>(x, n, bs, packed, scales, st);
  }
  return RQ_ERR_DTYPE;
}

template <int SDT>
static int nf4_deq_s(const uint8_t* p, int64_t nbytes, const void* s, int bs, void* out, int odt,
                     cudaStream_t st) {
  const int g = grid_1d((nbytes + 7) / 8);
  const PlainScales<SDT> sp{static_cast<const typename DType<SDT>::T*>(s)};
  const int64_t nv = 2 * nbytes;
  switch (odt) {
    case RQ_F32: nf4_dequantize_k<PlainScales<SDT>, RQ_F32><<<g, 256, 0, st>>>(p, nv, sp, bs, (float*)out); break;
    case RQ_BF16:
      nf4_dequantize_k<PlainScales<SDT>, RQ_BF16><<<g, 256, 0, st>>>(p, nv, sp, bs, (__nv_bfloat16*)out);
      break;
    case RQ_F16: nf4_dequantize_k<PlainScales<SDT>, RQ_F16><<<g, 256, 0, st>>>(p, nv, sp, bs, (__half*)out); break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

int nf4_dequantize(const uint8_t* p, int64_t nbytes, const void* s, int sdt, int bs, void* out, int odt,
                   cudaStream_t st) {
  switch (sdt) {
    case RQ_F32: return nf4_deq_s<RQ_F32>(p, nbytes, s, bs, out, odt, st);
    case RQ_BF16: return nf4_deq_s<RQ_BF16>(p, nbytes, s, bs, out, odt, st);
    case RQ_F16: return nf4_deq_s<RQ_F16>(p, nbytes, s, bs, out, odt, st);
  }
  return RQ_ERR_DTYPE;
}

int dq_dequantize(const uint8_t* p, int64_t numel, const uint8_t* c2, const float* c2s, int fp8, int bs,
                  int bs2, void* out, int odt, cudaStream_t st) {
  const int g = grid_1d((numel + 15) / 16);
  const DqScales sf{c2, c2s, fp8, bs2};
  switch (odt) {
    case RQ_F32: nf4_dequantize_k<DqScales, RQ_F32><<<g, 256, 0, st>>>(p, numel, sf, bs, (float*)out); break;
    case RQ_BF16:
      nf4_dequantize_k<DqScales, RQ_BF16><<<g, 256, 0, st>>>(p, numel, sf, bs, (__nv_bfloat16*)out);
      break;
    case RQ_F16: nf4_dequantize_k<DqScales, RQ_F16><<<g, 256, 0, st>>>(p, numel, sf, bs, (__half*)out); break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

int dq_quantize_scales(const float* c1, int64_t nb, int bs2, int fp8, uint8_t* c2, float* c2s, cudaStream_t st) {
  const int64_t ng = (nb + bs2 - 1) / bs2;
  dq_quantize_scales_k<<<grid_1d(ng * 32), 256, 0, st>>>(c1, nb, bs2, fp8, c2, c2s);
  return check_launch();
}

int int8_quantize(const void* x, int dtype, int64_t n, int bs, int8_t* q, void* scales, cudaStream_t st) {
  const int64_t nb = (n + bs - 1) / bs;
  const int g = grid_1d(nb * 32);
  switch (dtype) {
    case RQ_F32: int8_quantize_k<RQ_F32><<<g, 256, 0, st>>>((const float*)x, n, nb, bs, q, (float*)scales); break;
    case RQ_BF16:
      int8_quantize_k<RQ_BF16><<<g, 256, 0, st>>>((const __nv_bfloat16*)x, n, nb, bs, q, (__nv_bfloat16*)scales);
      break;
    case RQ_F16:
      int8_quantize_k<RQ_F16><<<g, 256, 0, st>>>((const __half*)x, n, nb, bs, q, (__half*)scales);
      break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

int int8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t cols, int8_t* q, void* scales,
                       cudaStream_t st) {
  if (rows > 0x7fffffff) return RQ_ERR_INVALID;
  switch (dtype) {
    case RQ_F32: int8_quantize_rows_k<RQ_F32><<<(int)rows, 256, 0, st>>>((const float*)x, cols, q, (float*)scales); break;
    case RQ_BF16:
      int8_quantize_rows_k<RQ_BF16><<<(int)rows, 256, 0, st>>>((const __nv_bfloat16*)x, cols, q,
                                                               (__nv_bfloat16*)scales);
      break;
    case RQ_F16:
      int8_quantize_rows_k<RQ_F16><<<(int)rows, 256, 0, st>>>((const __half*)x, cols, q, (__half*)scales);
      break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

template <int SDT>
static int int8_deq_s(const int8_t* q, int64_t n, const void* s, int bs, int64_t cols, void* out, int odt,
                      cudaStream_t st) {
  const int g = grid_1d((n + 15) / 16);
  const auto* sp = static_cast<const typename DType<SDT>::T*>(s);
  switch (odt) {
    case RQ_F32: int8_dequantize_k<SDT, RQ_F32><<<g, 256, 0, st>>>(q, n, sp, bs, cols, (float*)out); break;
    case RQ_BF16:
      int8_dequantize_k<SDT, RQ_BF16><<<g, 256, 0, st>>>(q, n, sp, bs, cols, (__nv_bfloat16*)out);
      break;
    case RQ_F16: int8_dequantize_k<SDT, RQ_F16><<<g, 256, 0, st>>>(q, n, sp, bs, cols, (__half*)out); break;
    default: return RQ_ERR_DTYPE;
  }
  return check_launch();
}

int int8_dequantize(const int8_t* q, int64_t n, const void* s, int sdt, int bs, int64_t cols, void* out, int odt,
                    cudaStream_t st) {
  switch (sdt) {
    case RQ_F32: return int8_deq_s<RQ_F32>(q, n, s, bs, cols, out, odt, st);
    case RQ_BF16: return int8_deq_s<RQ_BF16>(q, n, s, bs, cols, out, odt, st);
    case RQ_F16: return int8_deq_s<RQ_F16>(q, n, s, bs, cols, out, odt, st);
  }
  return RQ_ERR_DTYPE;
}

}  // namespace rq
