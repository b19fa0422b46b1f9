// gemv_kernels.cu -- decode-shaped (M <= 16) fused dequant + GEMV + LoRA,
// register-fed: the int8 formats where their rows cannot travel as the TMA
// ring's 128-byte pieces (K % 128 != 0, unaligned scales); every other decode
// call runs on the TMA-ring kernel of gemv_nf4.cu.  Also the dispatch of the
// decode path (gemv_forward, gemv_supported, gemv_fuse_down).
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

#include "gemv_common.cuh"

namespace rq {

constexpr int kGemvStageU = 16;  // scale loads issued per thread before use

// WK: 0 = NF4 family (table lookup, per-block scale), 1 = INT8 blockwise,
//     2 = INT8 per-row.  MT: 8 (M <= 8) or 16.  NT: 8-row tiles per chunk.
template <int DT, int WK, int MT, int NT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_k(const GemvArgs p) {
  using T = typename DType<DT>::T;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int N = (int)p.w.N, K = (int)p.w.K, M = (int)p.M;
  const int nbk = K / 64;
  constexpr int CH = NT * 8;
  constexpr int SCS = CH + 2;  // scale-table row stride (floats)

  uint32_t* lut = reinterpret_cast<uint32_t*>(smem);
  float* sc = reinterpret_cast<float*>(smem + (WK == 0 ? 256 * 32 * 4 : 0));
  float4* red = reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(sc) +
                                          (WK != 2 ? ((nbk * SCS * 4 + 15) / 16) * 16 : 0));
  T* tl = reinterpret_cast<T*>(red + kGemvWarps * NT * 32);  // staged x.A^T [M, r]

  if constexpr (WK == 0) {
    for (int i = tid; i < 256 * 32; i += kGemvThreads) {
      const int v = i >> 5;
      lut[i] = pack2<DT>(kNF4[v & 15], kNF4[v >> 4]);
    }
  }
  const uint32_t* lane4 = lut + lane;

  const int tile_begin = (int)((int64_t)p.tiles * blockIdx.x / p.grid);
  const int tile_end = (int)((int64_t)p.tiles * (blockIdx.x + 1) / p.grid);
  const int kb0 = nbk * warp / kGemvWarps, kb1 = nbk * (warp + 1) / kGemvWarps;
  const uint8_t* qb = static_cast<const uint8_t*>(p.w.q);
  const T* xp = static_cast<const T*>(p.x);
  const bool rowa = g < M, rowb = (MT == 16) && (g + 8 < M);
  const T* xa = xp + (size_t)(rowa ? g : 0) * K + t * 16;
  const T* xb = xp + (size_t)(rowb ? g + 8 : 0) * K + t * 16;
  constexpr int CW = (WK == 0) ? 2 : 4;   // 32-bit words of codes per lane per tile per block
  constexpr int RB = (WK == 0) ? 32 : 64; // code bytes per row per block

  const int ntot = tile_end - tile_begin;
  for (int ch = 0; ch < p.chunks; ++ch) {
    const int t0 = tile_begin + (int)((int64_t)ntot * ch / p.chunks);
    const int t1 = tile_begin + (int)((int64_t)ntot * (ch + 1) / p.chunks);
    const int ntiles = t1 - t0;
    const int c0 = t0 * 8;
    const int R = (t1 * 8 < N ? t1 * 8 : N) - c0;
    if (R <= 0) break;
    uint32_t roff[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int rl = nt * 8 + g;
      roff[nt] = rl < R ? (uint32_t)(c0 + rl) * (uint32_t)(nbk * RB) + t * (RB / 4) : 0xFFFFFFFFu;
    }
    auto load_codes = [&](int b, uint32_t (&dst)[NT][CW]) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt < ntiles && roff[nt] != 0xFFFFFFFFu) {
          const unsigned char* src = qb + roff[nt] + (uint32_t)b * RB;
          if constexpr (WK == 0) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(src));
            dst[nt][0] = v.x, dst[nt][1] = v.y;
          } else {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
            dst[nt][0] = v.x, dst[nt][1] = v.y, dst[nt][2] = v.z, dst[nt][3] = v.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < CW; ++i) dst[nt][i] = 0u;
        }
      }
    };
    auto load_x = [&](int b, uint32_t (&dst)[16]) {
      if (rowa) {
        const uint4* s = reinterpret_cast<const uint4*>(xa + b * 64);
        const uint4 u0 = __ldg(s), u1 = __ldg(s + 1);
        dst[0] = u0.x, dst[1] = u0.y, dst[2] = u0.z, dst[3] = u0.w, dst[4] = u1.x, dst[5] = u1.y, dst[6] = u1.z,
        dst[7] = u1.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = 0u;
      }
      if (rowb) {
        const uint4* s = reinterpret_cast<const uint4*>(xb + b * 64);
        const uint4 u0 = __ldg(s), u1 = __ldg(s + 1);
        dst[8] = u0.x, dst[9] = u0.y, dst[10] = u0.z, dst[11] = u0.w, dst[12] = u1.x, dst[13] = u1.y,
        dst[14] = u1.z, dst[15] = u1.w;
      } else {
#pragma unroll
        for (int i = 8; i < 16; ++i) dst[i] = 0u;
      }
    };

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

    // one block of MMAs for all tiles from (codes, x) register sets
    auto block_mma = [&](int b, const uint32_t (&cd)[NT][CW], const uint32_t (&xc)[16]) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt < ntiles) {
          float part[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t b0, b1;
            if constexpr (WK == 0) {
              const uint32_t word = cd[nt][j >> 1];
              if (j & 1) {
                b0 = lut_at<16>(word, lane4);
                b1 = lut_at<24>(word, lane4);
              } else {
                b0 = lut_at<0>(word, lane4);
                b1 = lut_at<8>(word, lane4);
              }
            } else {
              const uint32_t word = cd[nt][j];
              b0 = pack2<DT>((float)(int8_t)(word & 0xFF), (float)(int8_t)((word >> 8) & 0xFF));
              b1 = pack2<DT>((float)(int8_t)((word >> 16) & 0xFF), (float)(int8_t)(word >> 24));
            }
            if constexpr (WK == 2)
              Mma16816<DT>::run(acc[nt], xc[2 * j], xc[8 + 2 * j], xc[2 * j + 1], xc[8 + 2 * j + 1], b0, b1);
            else if (j == 0)
              Mma16816Zero<DT>::run(part, xc[0], xc[8], xc[1], xc[9], b0, b1);
            else
              Mma16816<DT>::run(part, xc[2 * j], xc[8 + 2 * j], xc[2 * j + 1], xc[8 + 2 * j + 1], b0, b1);
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
    };

    // NF4 keeps two blocks of codes in flight (ping-pong); INT8 (twice the
    // code bytes) loads each block where it is used.
    uint32_t cA[NT][CW], cB[NT][CW], xA[16], xB[16];
    if (kb0 < kb1) {
      if constexpr (WK == 0) load_codes(kb0, cA);
      load_x(kb0, xA);
    }
    if constexpr (WK != 2) {
      // each warp expands the scales of its own blocks for all rows of the
      // chunk (no CTA barrier needed); all loads of a round are issued
      // before any is used
      const int nbw = kb1 - kb0;
      const int total = R * nbw;
      const float inv = 1.0f / (float)(nbw > 0 ? nbw : 1);
      for (int base = lane; base < total; base += 32 * kGemvStageU) {
        float v[kGemvStageU];
        int rl[kGemvStageU], bb[kGemvStageU];
#pragma unroll
        for (int u = 0; u < kGemvStageU; ++u) {
          const int idx = base + u * 32;
          rl[u] = __float2int_rz(((float)idx + 0.5f) * inv);
          bb[u] = idx - rl[u] * nbw;
          v[u] = idx < total ? block_scale(p.w, (int64_t)(c0 + rl[u]) * nbk + kb0 + bb[u]) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kGemvStageU; ++u)
          if (base + u * 32 < total) sc[(kb0 + bb[u]) * SCS + rl[u]] = v[u];
      }
      __syncwarp();
    }
    if (ch == 0) __syncthreads();  // the code table is complete

    for (int b = kb0; b < kb1; b += 2) {
      const bool has2 = b + 1 < kb1;
      if (has2) {
        if constexpr (WK == 0) load_codes(b + 1, cB);
        load_x(b + 1, xB);
      }
      if constexpr (WK != 0) load_codes(b, cA);
      block_mma(b, cA, xA);
      if (!has2) break;
      if (b + 2 < kb1) {
        if constexpr (WK == 0) load_codes(b + 2, cA);
        load_x(b + 2, xA);
      }
      if constexpr (WK != 0) load_codes(b + 1, cB);
      block_mma(b + 1, cB, xB);
    }

#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      if (nt < ntiles)
        red[(warp * NT + nt) * 32 + lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    if (ch == 0) {
      // x.A^T comes from the down-product kernel launched just before; with
      // an adapter this kernel is its programmatic dependent and waits for
      // it only here, after streaming the first pass's weights (every other
      // input was written by kernels that finished before the down product
      // let this kernel launch)
      asm volatile("griddepcontrol.wait;" ::: "memory");
      if (p.r > 0) {
        const T* td = static_cast<const T*>(p.tdown);
        for (int i = tid; i < M * p.r; i += kGemvThreads) tl[i] = td[i];
      }
    }
    __syncthreads();

    const bool has_bias = p.bias != nullptr, has_lora = p.r > 0;
    const T* lb = static_cast<const T*>(p.lora_b);
    T* y = static_cast<T*>(p.y);
    for (int o = tid; o < CH * MT; o += kGemvThreads) {
      const int nl = o % CH, m = o / CH;
      if (nl >= R || m >= M) continue;
      const int nt = nl >> 3, cc = nl & 7, tt = cc >> 1, e = cc & 1;
      const int ln = (m & 7) * 4 + tt, comp = (m >> 3) * 2 + e;
      float sum = 0.0f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) {
        const float* rv = reinterpret_cast<const float*>(&red[(w * NT + nt) * 32 + ln]);
        sum += rv[comp];
      }
      const int row = c0 + nl;
      if constexpr (WK == 2) sum *= load_scalar(p.w.scales, p.w.sdt, row);
      float u = 0.0f;
      if (has_lora) {
        const T* brow = lb + (size_t)row * p.r;
        const T* trow = tl + m * p.r;
#pragma unroll 8
        for (int j = 0; j < p.r; ++j) u = fmaf(DType<DT>::to_f32(trow[j]), DType<DT>::to_f32(__ldg(brow + j)), u);
      }
      const float bv = has_bias ? load_scalar(p.bias, p.bdt, row) : 0.0f;
      y[(size_t)m * N + row] = DType<DT>::from_f32(lora_epilogue<DT>(sum, has_bias, bv, u, has_lora, p.s));
    }
    __syncthreads();
  }
}

// Shared memory the GEMV needs for this K, tile count and adapter size.
static size_t gemv_smem(int wk, int64_t K, int nt, int64_t M, int r) {
  size_t s = 0;
  if (wk == 0) s += 256 * 32 * 4;
  if (wk != 2) s += ((size_t)(K / 64) * (nt * 8 + 2) * 4 + 15) / 16 * 16;
  s += (size_t)kGemvWarps * nt * 32 * 16;
  s += (size_t)M * r * 2;
  return s;
}


static size_t smem_for(int wk, int64_t K, int nt, int64_t M, int r) {
  return gemv_smem(wk, K, nt, M, r);
}

// Launch shape: two CTAs per SM, each owning ceil(N/8)/grid whole 8-row
// tiles, processed in `chunks` passes of at most NT <= 8 tiles.  With an
// adapter the down-product kernel (one CTA on each of kLoraDownCtas SMs)
// runs beside this one: those SMs hold one GEMV CTA, so the grid leaves
// out one CTA for each (no CTA waits for a second wave).
static void gemv_shape(int wk, int64_t N, int64_t K, int64_t M, int r, int* grid, int* tiles, int* chunks,
                       int* nt) {
  const int64_t T = (N + 7) / 8;
  int64_t G = 2 * num_sms() - (r > 0 ? kLoraDownCtas : 0);
  if (G > T) G = T;
  const int64_t per = (T + G - 1) / G;
  int64_t ch = (per + kGemvMaxNT - 1) / kGemvMaxNT;
  int64_t n = (per + ch - 1) / ch;
  while (n > 1 && smem_for(wk, K, (int)n, M, r) > kGemvSmemCap) {
    ++ch;
    n = (per + ch - 1) / ch;
  }
  *grid = (int)G;
  *tiles = (int)T;
  *chunks = (int)ch;
  *nt = (int)n;
}

// Whether the TMA-ring GEMV (gemv_nf4.cu: NF4 formats, int8 with K % 128 == 0)
// can compute the layer's LoRA down product in its own grid (down_role): an
// adapter of rank <= 64, no fused gather,
// 4-byte aligned x_lora rows and A rows (K is a multiple of 64).
bool gemv_fuse_down(const LinearArgs& a) {
  const bool ring = is_nf4_fmt(a.w.fmt) || gemv_nf4_fits(a.w, a.M, a.r);  // the TMA-ring kernel runs the call
  return ring && a.r > 0 && a.r <= 64 && a.M >= 1 && a.M <= 16 && a.gather == nullptr &&
         a.lora_x != nullptr && a.lora_a != nullptr && ((uintptr_t)a.lora_x % 4) == 0 &&
         ((uintptr_t)a.lora_a % 4) == 0;
}

bool gemv_supported(const LinearArgs& a) {
  if (a.M < 1 || a.M > 16) return false;
  if (a.xdt != RQ_BF16 && a.xdt != RQ_F16) return false;
  if (a.w.K % 64 != 0 || a.w.bs != 64) return false;
  if ((uintptr_t)a.x % 16 || (uintptr_t)a.w.q % 16) return false;
  if (a.w.N > 0x7fffffff || a.w.K > 0x7fffffff || (a.w.N * a.w.K) / 2 > 0xfffffff0ll) return false;
  if (is_nf4_fmt(a.w.fmt)) return gemv_nf4_fits(a.w, a.M, a.r);
  if (gemv_nf4_fits(a.w, a.M, a.r)) return true;  // int8 on the TMA-ring kernel
  const int wk = a.w.fmt == RQ_W_INT8 ? 1 : 2;
  return smem_for(wk, a.w.K, 1, a.M, a.r) <= kGemvSmemCap;
}

template <int DT, int WK, int MT, int NT>
static int gemv_launch(const GemvArgs& g, size_t smem, cudaStream_t st) {
  auto kern = gemv_k<DT, WK, MT, NT>;
  const int rc = ensure_smem_limit((const void*)kern, smem);
  if (rc != RQ_OK) return rc;
  // with an adapter: the programmatic dependent of the down-product kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g.grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g.r > 0 ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return check_launch();
}

template <int DT, int WK, int MT>
static int gemv_nt(const GemvArgs& g, int nt, size_t smem, cudaStream_t st) {
  return nt <= 4 ? gemv_launch<DT, WK, MT, 4>(g, smem, st) : gemv_launch<DT, WK, MT, 8>(g, smem, st);
}

template <int DT>
static int gemv_dt(const GemvArgs& g, int wk, int nt, size_t smem, cudaStream_t st) {
  const bool m16 = g.M > 8;
  if (wk == 1) return m16 ? gemv_nt<DT, 1, 16>(g, nt, smem, st) : gemv_nt<DT, 1, 8>(g, nt, smem, st);
  return m16 ? gemv_nt<DT, 2, 16>(g, nt, smem, st) : gemv_nt<DT, 2, 8>(g, nt, smem, st);
}

int gemv_forward(const LinearArgs& a, const void* tdown, cudaStream_t st, float* partial, unsigned* counters) {
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
  g.xdt = a.xdt;
  g.gather = a.gather != nullptr;
  if (a.gather) g.gth = *a.gather;
  // with `partial` the NF4 GEMV computes tdown itself (gemv_fuse_down)
  g.fuse_down = partial != nullptr;
  g.lora_x = a.lora_x;
  g.lora_a = a.lora_a;
  g.partial = partial;
  g.counters = counters;
  if (is_nf4_fmt(a.w.fmt)) return gemv_nf4_forward(g, a.r > 0, st);
  if (a.gather) return RQ_ERR_UNSUPPORTED;  // int8: no fused gather
  // int8 rows that travel as 128-byte pieces: the TMA-ring kernel (gemv_nf4.cu)
  if (gemv_nf4_fits(a.w, a.M, a.r)) return gemv_nf4_forward(g, a.r > 0, st);
  const int wk = a.w.fmt == RQ_W_INT8 ? 1 : 2;
  int nt = 1;
  gemv_shape(wk, a.w.N, a.w.K, a.M, a.r, &g.grid, &g.tiles, &g.chunks, &nt);
  nt = nt <= 4 ? 4 : 8;
  g.chunks = (int)(((g.tiles + g.grid - 1) / g.grid + nt - 1) / nt);
  const size_t smem = gemv_smem(wk, a.w.K, nt, a.M, a.r);
  return a.xdt == RQ_BF16 ? gemv_dt<RQ_BF16>(g, wk, nt, smem, st) : gemv_dt<RQ_F16>(g, wk, nt, smem, st);
}

}  // namespace rq
