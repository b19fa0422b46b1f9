// linear_common.cuh -- device-side views and the exact epilogue shared by
// the QuantLinear+LoRA kernels (GEMV, tcgen05 GEMM, SIMT).
#pragma once

#include "rq_common.cuh"
#include "rq_internal.h"

namespace rq {

constexpr int kDQBlock2 = 256;  // second-level block of QuantLinear.enable_double_quant

__device__ __forceinline__ float load_scalar(const void* p, int dt, int64_t i) {
  switch (dt) {
    case RQ_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case RQ_F16: return __half2float(static_cast<const __half*>(p)[i]);
    default: return static_cast<const float*>(p)[i];
  }
}

// First-level scale of block b, exactly as the reference reconstructs it:
// NF4/INT8: the stored scale promoted to fp32; DQ: c2 (fp8 or int8/127)
// times c2_scales (double_quant.py:106-111).
__device__ __forceinline__ float block_scale(const QWeight& w, int64_t b) {
  switch (w.fmt) {
    case RQ_W_NF4_DQ_FP8: return e4m3fnuz_to_f32(w.c2[b]) * w.c2s[b / kDQBlock2];
    case RQ_W_NF4_DQ_INT8: return ieee_div((float)(int8_t)w.c2[b], 127.0f) * w.c2s[b / kDQBlock2];
    default: return load_scalar(w.scales, w.sdt, b);
  }
}

// Dequantized fp32 value of flat weight element `flat` (row n = flat / K),
// the value dequantize_int4 / dequantize_int8 / double_dequantize produce.
__device__ __forceinline__ float deq_elem(const QWeight& w, int64_t flat, const float* lut16) {
  if (is_nf4_fmt(w.fmt)) {
    const uint8_t byte = static_cast<const uint8_t*>(w.q)[flat >> 1];
    const int code = (flat & 1) ? (byte >> 4) : (byte & 0xF);
    return lut16[code] * block_scale(w, flat / w.bs);
  }
  const float q = (float)static_cast<const int8_t*>(w.q)[flat];
  const int64_t si = w.fmt == RQ_W_INT8_ROW ? flat / w.K : flat / w.bs;
  return q * load_scalar(w.scales, w.sdt, si);
}

// The rounding sequence of LoRALinear.forward over QuantLinear.forward in
// the activation dtype (lora_layer.py:63-70, quant_linear.py:196-197):
//   base = rnd(acc + rnd(bias));  u = rnd(t . b_row);  v = rnd(u * s);
//   y = rnd(base + v).
template <int DT>
__device__ __forceinline__ float lora_epilogue(float acc, bool has_bias, float bias_v, float u_acc, bool has_lora,
                                               float s) {
  float base = has_bias ? round_to<DT>(acc + round_to<DT>(bias_v)) : round_to<DT>(acc);
  if (!has_lora) return base;
  const float u = round_to<DT>(u_acc);
  const float v = round_to<DT>(u * s);
  return round_to<DT>(base + v);
}

}  // namespace rq
