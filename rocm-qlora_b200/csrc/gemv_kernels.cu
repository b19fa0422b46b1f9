// gemv_kernels.cu -- decode-shaped (M <= 16) fused dequant + GEMV + LoRA.
//
// Y[M, N] = X[M, K] . deq(W[N, K])^T, with the LoRA / bias epilogue of
// LoRALinear.forward.  The weight stream dominates (N*K/2 bytes of NF4 codes
// against 2*M*K bytes of X), so the kernel is built to keep HBM busy:
//
//  * one CTA per SM (16 warps), each CTA owns a contiguous range of ~N/148
//    output rows, so every SM streams the same number of code bytes;
//  * the 16 warps split K (whole 64-element blocks) and keep fp32
//    accumulators for up to 64 rows; partial sums meet in shared memory in a
//    fixed order (deterministic);
//  * the tensor cores do the multiply: mma.sync m16n8k16 with X as the A
//    operand (the M <= 16 tokens are its 16 rows) and 8 weight rows as B;
//  * NF4 codes become 16-bit operands through a 256-entry shared-memory
//    table indexed by the code byte (two levels per lookup), replicated 32x
//    so each lane reads its own bank;
//  * the per-block scale is applied to the fp32 partial product of each
//    64-wide block (acc += s_b * sum_{k in b} x_k T[c_k]); scales (including
//    the fp8 double-quant decode) are expanded once per CTA into shared
//    memory.
//
// Numerics: the reference rounds each dequantized weight T[c]*s to the
// activation dtype before its matmul; here T[c] is rounded instead and s is
// applied in fp32.  Both are one rounding of the same size per weight, and
// the output stays within the parity tolerance (tests/tolerance.py).
#include <cuda_runtime.h>

#include "linear_common.cuh"

namespace rq {

template <int DT> struct Mma16816;
template <> struct Mma16816<RQ_BF16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct Mma16816<RQ_F16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

constexpr int kGemvWarps = 16;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvNT = 8;  // n-tiles of 8 rows held per warp (64 rows)

struct GemvArgs {
  QWeight w;
  const void* x;
  int64_t M;
  const void* bias;
  int bdt;
  const void* tdown;   // [M, r] rounded x.A^T, activation dtype
  const void* lora_b;  // [N, r]
  int r;
  float s;
  void* y;
  int chunk_rows;      // 64 or 32
  int grid;
};

// WK: 0 = NF4 family (table lookup, per-block scale), 1 = INT8 blockwise,
//     2 = INT8 per-row.  MT: 8 (M <= 8) or 16.
template <int DT, int WK, int MT>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_k(const GemvArgs p) {
  using T = typename DType<DT>::T;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t N = p.w.N, K = p.w.K, M = p.M;
  const int64_t nbk = K / 64;
  const int CH = p.chunk_rows;
  const int SCS = CH + 2;  // scale-table row stride (floats)

  uint32_t* lut = reinterpret_cast<uint32_t*>(smem);
  float* sc = reinterpret_cast<float*>(smem + (WK == 0 ? 256 * 32 * 4 : 0));
  float4* red = reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(sc) +
                                          (WK != 2 ? ((nbk * SCS * 4 + 15) / 16) * 16 : 0));

  if constexpr (WK == 0) {
    for (int i = tid; i < 256 * 32; i += kGemvThreads) {
      const int v = i >> 5;
      lut[i] = pack2<DT>(kNF4[v & 15], kNF4[v >> 4]);
    }
  }

  const int64_t r_begin = N * blockIdx.x / p.grid;
  const int64_t r_end = N * (blockIdx.x + 1) / p.grid;
  const int64_t kb0 = nbk * warp / kGemvWarps, kb1 = nbk * (warp + 1) / kGemvWarps;
  const uint8_t* qb = static_cast<const uint8_t*>(p.w.q);
  const T* xp = static_cast<const T*>(p.x);
  const bool rowa = g < M, rowb = (MT == 16) && (g + 8 < M);
  const T* xa = xp + (rowa ? g : 0) * K;
  const T* xb = xp + (rowb ? g + 8 : 0) * K;

  for (int64_t c0 = r_begin; c0 < r_end; c0 += CH) {
    const int R = (int)(r_end - c0 < CH ? r_end - c0 : CH);
    const int ntiles = (R + 7) >> 3;
    if constexpr (WK != 2) {
      for (int64_t i = tid; i < (int64_t)R * nbk; i += kGemvThreads) {
        const int64_t rl = i / nbk, b = i % nbk;
        sc[b * SCS + rl] = block_scale(p.w, (c0 + rl) * nbk + b);
      }
      for (int64_t i = tid; i < (int64_t)(CH - R) * nbk; i += kGemvThreads) {
        const int64_t rl = R + i / nbk, b = i % nbk;
        sc[b * SCS + rl] = 0.0f;
      }
    }
    __syncthreads();

    float acc[kGemvNT][4];
#pragma unroll
    for (int i = 0; i < kGemvNT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

    // code bytes per lane per n-tile per block: NF4 8 bytes, INT8 16 bytes
    constexpr int CW = (WK == 0) ? 2 : 4;  // 32-bit words
    uint32_t cur[kGemvNT][CW];
    auto load_codes = [&](int64_t b, uint32_t (&dst)[kGemvNT][CW]) {
#pragma unroll
      for (int nt = 0; nt < kGemvNT; ++nt) {
        const int rl = nt * 8 + g;
        if (nt < ntiles && rl < R) {
          const int64_t row = c0 + rl;
          if constexpr (WK == 0) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(qb + row * (K / 2) + b * 32 + t * 8));
            dst[nt][0] = v.x;
            dst[nt][1] = v.y;
          } else {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(qb + row * K + b * 64 + t * 16));
            dst[nt][0] = v.x;
            dst[nt][1] = v.y;
            dst[nt][2] = v.z;
            dst[nt][3] = v.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < CW; ++i) dst[nt][i] = 0u;
        }
      }
    };
    // NF4: prefetch the next block's codes; INT8 (twice the bytes) loads in place
    constexpr bool kPrefetch = (WK == 0);
    if (kPrefetch && kb0 < kb1) load_codes(kb0, cur);

    for (int64_t b = kb0; b < kb1; ++b) {
      uint32_t nxt[kGemvNT][CW];
      if (kPrefetch) {
        if (b + 1 < kb1) load_codes(b + 1, nxt);
      } else {
        load_codes(b, cur);
      }
      // X fragments: 16 consecutive k per lane, rows g and g+8
      uint32_t xa_r[8], xb_r[8];
      {
        if (rowa) {
          const uint4* s = reinterpret_cast<const uint4*>(xa + b * 64 + t * 16);
          const uint4 u0 = __ldg(s), u1 = __ldg(s + 1);
          xa_r[0] = u0.x, xa_r[1] = u0.y, xa_r[2] = u0.z, xa_r[3] = u0.w;
          xa_r[4] = u1.x, xa_r[5] = u1.y, xa_r[6] = u1.z, xa_r[7] = u1.w;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) xa_r[i] = 0u;
        }
        if (rowb) {
          const uint4* s = reinterpret_cast<const uint4*>(xb + b * 64 + t * 16);
          const uint4 u0 = __ldg(s), u1 = __ldg(s + 1);
          xb_r[0] = u0.x, xb_r[1] = u0.y, xb_r[2] = u0.z, xb_r[3] = u0.w;
          xb_r[4] = u1.x, xb_r[5] = u1.y, xb_r[6] = u1.z, xb_r[7] = u1.w;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) xb_r[i] = 0u;
        }
      }
#pragma unroll
      for (int nt = 0; nt < kGemvNT; ++nt) {
        if (nt < ntiles) {
          float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t b0, b1;
            if constexpr (WK == 0) {
              const uint32_t word = cur[nt][j >> 1];
              const uint32_t v0 = (word >> (16 * (j & 1))) & 0xFFu;
              const uint32_t v1 = (word >> (16 * (j & 1) + 8)) & 0xFFu;
              b0 = lut[(v0 << 5) | lane];
              b1 = lut[(v1 << 5) | lane];
            } else {
              const uint32_t word = cur[nt][j];
              b0 = pack2<DT>((float)(int8_t)(word & 0xFF), (float)(int8_t)((word >> 8) & 0xFF));
              b1 = pack2<DT>((float)(int8_t)((word >> 16) & 0xFF), (float)(int8_t)(word >> 24));
            }
            if constexpr (WK == 2)
              Mma16816<DT>::run(acc[nt], xa_r[2 * j], xb_r[2 * j], xa_r[2 * j + 1], xb_r[2 * j + 1], b0, b1);
            else
              Mma16816<DT>::run(part, xa_r[2 * j], xb_r[2 * j], xa_r[2 * j + 1], xb_r[2 * j + 1], b0, b1);
          }
          if constexpr (WK != 2) {
            const float2 s2 = *reinterpret_cast<const float2*>(&sc[b * SCS + nt * 8 + 2 * t]);
            acc[nt][0] = fmaf(part[0], s2.x, acc[nt][0]);
            acc[nt][1] = fmaf(part[1], s2.y, acc[nt][1]);
            acc[nt][2] = fmaf(part[2], s2.x, acc[nt][2]);
            acc[nt][3] = fmaf(part[3], s2.y, acc[nt][3]);
          }
        }
      }
      if (kPrefetch && b + 1 < kb1) {
#pragma unroll
        for (int nt = 0; nt < kGemvNT; ++nt)
#pragma unroll
          for (int i = 0; i < CW; ++i) cur[nt][i] = nxt[nt][i];
      }
    }

#pragma unroll
    for (int nt = 0; nt < kGemvNT; ++nt)
      if (nt < ntiles) red[(warp * kGemvNT + nt) * 32 + lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    __syncthreads();

    const bool has_bias = p.bias != nullptr, has_lora = p.r > 0;
    const T* td = static_cast<const T*>(p.tdown);
    const T* lb = static_cast<const T*>(p.lora_b);
    T* y = static_cast<T*>(p.y);
    for (int o = tid; o < CH * MT; o += kGemvThreads) {
      const int nl = o % CH, m = o / CH;
      if (nl >= R || m >= M) continue;
      const int nt = nl >> 3, cc = nl & 7, tt = cc >> 1, e = cc & 1;
      const int ln = (m & 7) * 4 + tt, comp = (m >> 3) * 2 + e;
      float sum = 0.0f;
#pragma unroll 4
      for (int w = 0; w < kGemvWarps; ++w) {
        const float* rv = reinterpret_cast<const float*>(&red[(w * kGemvNT + nt) * 32 + ln]);
        sum += rv[comp];
      }
      const int64_t row = c0 + nl;
      if constexpr (WK == 2) sum *= load_scalar(p.w.scales, p.w.sdt, row);
      float u = 0.0f;
      if (has_lora)
        for (int j = 0; j < p.r; ++j)
          u = fmaf(DType<DT>::to_f32(td[m * p.r + j]), DType<DT>::to_f32(lb[row * p.r + j]), u);
      const float bv = has_bias ? load_scalar(p.bias, p.bdt, row) : 0.0f;
      y[m * N + row] = DType<DT>::from_f32(lora_epilogue<DT>(sum, has_bias, bv, u, has_lora, p.s));
    }
    __syncthreads();
  }
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

// Shared memory the GEMV needs for this K and chunk height.
static size_t gemv_smem(int wk, int64_t K, int chunk) {
  size_t s = 0;
  if (wk == 0) s += 256 * 32 * 4;
  if (wk != 2) s += ((size_t)(K / 64) * (chunk + 2) * 4 + 15) / 16 * 16;
  s += (size_t)kGemvWarps * kGemvNT * 32 * 16;
  return s;
}

bool gemv_supported(const LinearArgs& a) {
  if (a.M < 1 || a.M > 16) return false;
  if (a.xdt != RQ_BF16 && a.xdt != RQ_F16) return false;
  if (a.w.K % 64 != 0 || a.w.bs != 64) return false;
  if ((uintptr_t)a.x % 16 || (uintptr_t)a.w.q % 16) return false;
  const int wk = is_nf4_fmt(a.w.fmt) ? 0 : (a.w.fmt == RQ_W_INT8 ? 1 : 2);
  return gemv_smem(wk, a.w.K, 32) <= 227 * 1024;
}

template <int DT, int WK, int MT>
static int gemv_launch(const GemvArgs& g, size_t smem, cudaStream_t st) {
  auto kern = gemv_k<DT, WK, MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  kern<<<g.grid, kGemvThreads, smem, st>>>(g);
  return check_launch();
}

template <int DT>
static int gemv_dt(const GemvArgs& g, int wk, size_t smem, cudaStream_t st) {
  const bool m16 = g.M > 8;
  switch (wk) {
    case 0: return m16 ? gemv_launch<DT, 0, 16>(g, smem, st) : gemv_launch<DT, 0, 8>(g, smem, st);
    case 1: return m16 ? gemv_launch<DT, 1, 16>(g, smem, st) : gemv_launch<DT, 1, 8>(g, smem, st);
    default: return m16 ? gemv_launch<DT, 2, 16>(g, smem, st) : gemv_launch<DT, 2, 8>(g, smem, st);
  }
}

int gemv_forward(const LinearArgs& a, const void* tdown, cudaStream_t st) {
  GemvArgs g;
  g.w = a.w;
  g.x = a.x;
  g.M = a.M;
  g.bias = a.bias;
  g.bdt = a.bdt;
  g.tdown = tdown;
  g.lora_b = a.lora_b;
  g.r = a.r;
  g.s = a.scaling;
  g.y = a.y;
  const int wk = is_nf4_fmt(a.w.fmt) ? 0 : (a.w.fmt == RQ_W_INT8 ? 1 : 2);
  g.chunk_rows = gemv_smem(wk, a.w.K, 64) <= 227 * 1024 ? 64 : 32;
  const int64_t sms = num_sms();
  int64_t grid = sms;
  if (grid * 8 > a.w.N) grid = (a.w.N + 7) / 8;
  g.grid = (int)grid;
  const size_t smem = gemv_smem(wk, a.w.K, g.chunk_rows);
  return a.xdt == RQ_BF16 ? gemv_dt<RQ_BF16>(g, wk, smem, st) : gemv_dt<RQ_F16>(g, wk, smem, st);
}

}  // namespace rq
