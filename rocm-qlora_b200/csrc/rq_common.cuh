// rq_common.cuh -- device helpers shared by the rocm-qlora B200 kernels.
//
// Arithmetic here reproduces torch's CPU semantics for the quantization
// path of rocm_qlora (quant_ops.py, double_quant.py) bit for bit:
//   * bf16/f16 tensor ops compute in fp32 and round to nearest even;
//   * division is IEEE (div.rn.f32), never the fast approximate form;
//   * the NF4 nearest-level search is the 16-way fp32 argmin (first minimum
//     wins), evaluated through 15 exact decision thresholds;
//   * float -> int8 keeps the low byte of the truncated integer, NaN/inf -> 0;
//   * float8_e4m3fnuz is round-to-nearest-even, 0x80 = NaN, no -0.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/rq_b200.h"

namespace rq {

// NF4 levels (quant_ops.py:10-15), the double literals rounded to fp32.
__device__ __constant__ float kNF4[16] = {
    (float)-1.0, (float)-0.6961928009986877, (float)-0.5250730514526367, (float)-0.39491748809814453,
    (float)-0.28444138169288635, (float)-0.18477343022823334, (float)-0.09105003625154495, (float)0.0,
    (float)0.07958029955625534, (float)0.16093020141124725, (float)0.24611230194568634,
    (float)0.33791524171829224, (float)0.44070982933044434, (float)0.5626170039176941,
    (float)0.7229568362236023, (float)1.0};

// t[j] = the largest fp32 n with fl(|n-T_j|) <= fl(|n-T_{j+1}|); the argmin
// equals #{j : n > t[j]} for every fp32 n in [-1, 1] and for NaN (code 0).
// Verified exhaustively over all 2^31 such bit patterns on the CPU.
__device__ __forceinline__ int nf4_code(float n) {
  const float t0 = __uint_as_float(0xbf591cd9u), t1 = __uint_as_float(0xbf1c5271u),
              t2 = __uint_as_float(0xbeeb8480u), t3 = __uint_as_float(0xbeadea77u),
              t4 = __uint_as_float(0xbe703cedu), t5 = __uint_as_float(0xbe0d38bcu),
              t6 = __uint_as_float(0xbd3a7871u), t7 = __uint_as_float(0x3d22faffu),
              t8 = __uint_as_float(0x3df64862u), t9 = __uint_as_float(0x3e5067e0u),
              t10 = __uint_as_float(0x3e9582d4u), t11 = __uint_as_float(0x3ec753f9u),
              t12 = __uint_as_float(0x3f006d03u), t13 = __uint_as_float(0x3f248dafu),
              t14 = __uint_as_float(0x3f5c89d9u);
  // branch-free binary search over the sorted thresholds
  const bool b3 = n > t7;
  const float ta = b3 ? t11 : t3;
  const bool b2 = n > ta;
  const float tb = b3 ? (b2 ? t13 : t9) : (b2 ? t5 : t1);
  const bool b1 = n > tb;
  const float tc = b3 ? (b2 ? (b1 ? t14 : t12) : (b1 ? t10 : t8))
                      : (b2 ? (b1 ? t6 : t4) : (b1 ? t2 : t0));
  const bool b0 = n > tc;
  // NaN: every comparison is false -> 0, as torch.argmin returns the first NaN.
  return (b3 << 3) | (b2 << 2) | (b1 << 1) | (int)b0;
}

// ---------------------------------------------------------------- dtypes

template <int DT> struct DType;
template <> struct DType<RQ_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f32(T v) { return v; }
  static __device__ __forceinline__ T from_f32(float v) { return v; }
};
template <> struct DType<RQ_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f32(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f32(float v) { return __float2bfloat16_rn(v); }
};
template <> struct DType<RQ_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f32(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f32(float v) { return __float2half_rn(v); }
};

// Two fp32 values rounded to a 16-bit dtype, packed low | high << 16.
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (DT == RQ_BF16) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
  } else {
    return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
  }
}

// The value a torch tensor of dtype DT holds after an fp32 op.
template <int DT>
__device__ __forceinline__ float round_to(float v) {
  return DType<DT>::to_f32(DType<DT>::from_f32(v));
}

// torch.clamp(t, min=1e-12) in t's dtype; NaN passes through.
template <int DT>
__device__ __forceinline__ float clamp_eps(float v) {
  const float lo = round_to<DT>(1e-12f);
  return v < lo ? lo : v;  // NaN < lo is false -> NaN kept
}

__device__ __forceinline__ float ieee_div(float a, float b) { return __fdiv_rn(a, b); }

// float -> int8 as torch's CPU cast does it.
__device__ __forceinline__ int8_t to_int8_torch(float v) {
  if (!(fabsf(v) < 9.2233720368547758e18f)) return 0;  // NaN, inf, huge
  return (int8_t)(uint8_t)((unsigned long long)(long long)v & 0xFFull);
}

// float8_e4m3fnuz (bias 8, 3 mantissa bits, 0x80 = NaN, max 240).
__device__ __forceinline__ float e4m3fnuz_to_f32(uint32_t v) {
  v &= 0xFFu;
  if (v == 0x80u) return __uint_as_float(0x7fc00000u);
  const uint32_t e = (v >> 3) & 0xFu, m = v & 7u;
  float r = e == 0 ? (float)m * 0x1p-10f : __int_as_float((int)((e + 119u) << 23 | (m << 20)));
  return (v & 0x80u) ? -r : r;
}

__device__ __forceinline__ uint8_t f32_to_e4m3fnuz(float f) {
  if (isnan(f)) return 0x80;
  const uint32_t sign = (__float_as_uint(f) >> 24) & 0x80u;
  const float a = fabsf(f);
  if (isinf(a)) return 0x80;
  uint32_t code;
  if (a < 0x1p-7f) {
    code = (uint32_t)rintf(a * 1024.0f);  // subnormal step 2^-10, 8 -> 2^-7
  } else {
    int e = (int)((__float_as_uint(a) >> 23) & 0xFF) - 127;  // a is normal here
    const float m = __int_as_float((int)((__float_as_uint(a) & 0x7FFFFFu) | 0x3F800000u)) - 1.0f;
    uint32_t q = (uint32_t)rintf(m * 8.0f);
    int E = e + 8;
    if (q == 8u) { q = 0; E += 1; }
    if (E > 15) return 0x80;
    code = ((uint32_t)E << 3) | q;
  }
  if (code == 0) return 0x00;
  return (uint8_t)(sign | code);
}

// Warp-segment reductions over `L` consecutive lanes (L a power of two <= 32).
template <int L>
__device__ __forceinline__ float seg_max(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int L>
__device__ __forceinline__ bool seg_any(bool b) {
  unsigned m = __ballot_sync(0xffffffffu, b);
  const int lane = threadIdx.x & 31;
  const unsigned seg = (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (lane & ~(L - 1)));
  return (m & seg) != 0u;
}

}  // namespace rq
