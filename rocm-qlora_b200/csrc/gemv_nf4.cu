// gemv_nf4.cu -- decode-shaped (M <= 16) fused NF4 dequant + GEMV + LoRA.
//
// Y[M, N] = X[M, K] . deq(W[N, K])^T with the LoRA / bias epilogue of
// LoRALinear.forward, for NF4 weights with per-block scales or with
// double-quantized (fp8 e4m3fnuz or int8) scales.
//
// The code stream is the cost (N*K/2 bytes against 2*M*K bytes of X), so it
// is moved the way HBM likes it:
//
//  * two CTAs per SM; CTA i owns whole 8-row tiles [T*i/G, T*(i+1)/G), i.e.
//    one contiguous byte range of the weight (rows are contiguous);
//  * that range streams through a 4-stage shared-memory ring with bulk
//    asynchronous copies (cp.async.bulk, one per row and stage, 256 bytes =
//    8 blocks of 64 codes), completed on an mbarrier per stage; consumers
//    release a stage through a second mbarrier before it is refilled;
//  * the 8 warps of the CTA take one 64-block of every stage each, hold fp32
//    accumulators for all of the CTA's rows, and meet in shared memory at the
//    end in a fixed order (deterministic);
//  * the multiply runs on the tensor cores (mma.sync m16n8k16: X as the
//    16-row A operand, 8 weight rows as B); code bytes become 16-bit operand
//    pairs through a 256-entry shared table replicated 32x (one bank per
//    lane); the block scale multiplies each block's fp32 partial;
//  * scales are read one stage ahead per warp (one row per lane), decoded
//    through a 256-entry fp8/int8 table, and handed to the lanes that need
//    them with register shuffles.
//
// All waits are bounded.  A wait that runs out raises the CTA's abort flag
// (every later wait then returns at once, so the kernel finishes) and
// counts in a device counter read by rq_take_kernel_timeouts().
#include <cuda_runtime.h>

#include "gemv_common.cuh"

namespace rq {

constexpr int kNf4MaxStages = 16;
constexpr size_t kNf4RingBudget = 72 * 1024;  // ring bytes per CTA (two CTAs per SM)
constexpr int kStageBlocks = kGemvWarps;            // one 64-block per warp per stage
constexpr int kRowBytes = kStageBlocks * 32;         // code bytes per row per stage
constexpr int kRowStride = kRowBytes + 32;           // padded: conflict-free 8-byte reads
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ unsigned int g_kernel_timeouts;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Waits for the phase of `bar` with the given parity to complete, at most
// kWaitLimit polls; returns false (and raises the abort flag) if it gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (*abort_flag) return false;
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  *abort_flag = 1;
  atomicAdd(&g_kernel_timeouts, 1u);
  return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Ring slots for a tile count: as many stages as the budget holds (the whole
// K range when it fits), at least 2.
int gemv_nf4_stages(int nt, int64_t K) {
  const int64_t nst = (K / 64 + kStageBlocks - 1) / kStageBlocks;
  int64_t s = (int64_t)(kNf4RingBudget / ((size_t)nt * 8 * kRowStride));
  if (s > kNf4MaxStages) s = kNf4MaxStages;
  if (s > nst) s = nst;
  if (s < 2) s = 2;
  return (int)s;
}

size_t gemv_nf4_smem(int nt, int64_t K, int64_t M, int r) {
  const int S = gemv_nf4_stages(nt, K);
  return 256 * 32 * 4                                   // code-byte table
         + (size_t)S * nt * 8 * kRowStride              // ring (the reduction reuses it)
         + 256 * 4                                      // fp8 / int8 scale table
         + 2 * kNf4MaxStages * 8                        // mbarriers
         + (size_t)M * r * 2;                           // staged x.A^T
}

template <int DT, int MT, int NT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_nf4_k(const __grid_constant__ GemvArgs p) {
  using T = typename DType<DT>::T;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ int abort_flag;
  constexpr int CH = NT * 8;
  constexpr int STAGE = CH * kRowStride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int N = (int)p.w.N, K = (int)p.w.K, M = (int)p.M;
  const int nbk = K / 64;
  const int nst = (nbk + kStageBlocks - 1) / kStageBlocks;
  const int fmt = p.w.fmt;
  const bool dq = fmt != RQ_W_NF4;
  const uint32_t S = (uint32_t)p.stages;

  uint32_t* lut = reinterpret_cast<uint32_t*>(smem);
  unsigned char* ring = smem + 256 * 32 * 4;
  float* sclut = reinterpret_cast<float*>(ring + S * STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sclut + 256);  // full[S], empty[S]
  T* tl = reinterpret_cast<T*>(bars + 2 * kNf4MaxStages);
  float4* red = reinterpret_cast<float4*>(ring);  // after the main loop
  const uint32_t ring_s = smem_addr(ring);
  const uint32_t full0 = smem_addr(bars), empty0 = full0 + kNf4MaxStages * 8;

  if (tid == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kGemvWarps);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t* lut_lane = lut + lane;

  const int tile_begin = (int)((int64_t)p.tiles * blockIdx.x / p.grid);
  const int tile_end = (int)((int64_t)p.tiles * (blockIdx.x + 1) / p.grid);
  const int ntot = tile_end - tile_begin;
  const uint8_t* qb = static_cast<const uint8_t*>(p.w.q);
  const T* xp = static_cast<const T*>(p.x);
  const bool rowa = g < M, rowb = (MT == 16) && (g + 8 < M);
  const T* xa = xp + (size_t)(rowa ? g : 0) * K + t * 16;
  const T* xb = xp + (size_t)(rowb ? g + 8 : 0) * K + t * 16;
  volatile int* abortp = &abort_flag;

  uint32_t gs = 0;  // stages issued / consumed before this chunk (ring slot and phase)
  for (int ch = 0; ch < p.chunks; ++ch) {
    const int t0 = tile_begin + (int)((int64_t)ntot * ch / p.chunks);
    const int t1 = tile_begin + (int)((int64_t)ntot * (ch + 1) / p.chunks);
    const int ntiles = t1 - t0;
    const int c0 = t0 * 8;
    const int R = (t1 * 8 < N ? t1 * 8 : N) - c0;
    if (R <= 0) break;

    // producer (warp 0): stage s of this chunk = blocks [8s, 8s+8) of rows
    // c0..c0+R-1, one bulk copy per row
    auto issue = [&](int s) {
      const uint32_t gst = gs + s, slot = gst % S;
      if (gst >= S && !mbar_wait(empty0 + 8 * slot, ((gst / S) + 1) & 1, abortp)) return;
      const int nbs = nbk - s * kStageBlocks < kStageBlocks ? nbk - s * kStageBlocks : kStageBlocks;
      const uint32_t bytes = (uint32_t)nbs * 32;
      if (lane == 0) mbar_expect_tx(full0 + 8 * slot, bytes * (uint32_t)R);
      __syncwarp();
      for (int rl = lane; rl < R; rl += 32)
        bulk_g2s(ring_s + slot * STAGE + rl * kRowStride,
                 qb + (size_t)(c0 + rl) * (size_t)(K / 2) + (size_t)s * kRowBytes, bytes, full0 + 8 * slot);
    };
    if (warp == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // ring was written by threads (reduction)
      for (int s = 0; s < (int)S - 1 && s < nst; ++s) issue(s);
    }
    if (ch == 0) {
      // tables, built while the first stages are in flight: each thread makes
      // one code-byte entry, the warp writes the 32 copies of its 32 entries
      const uint32_t mine = pack2<DT>(kNF4[tid & 15], kNF4[tid >> 4]);
#pragma unroll 8
      for (int j = 0; j < 32; ++j) lut[((warp * 32 + j) << 5) | lane] = __shfl_sync(0xffffffffu, mine, j);
      if (dq) sclut[tid] = fmt == RQ_W_NF4_DQ_FP8 ? e4m3fnuz_to_f32(tid) : ieee_div((float)(int8_t)tid, 127.0f);
      if (p.r > 0) {
        const T* td = static_cast<const T*>(p.tdown);
        for (int i = tid; i < M * p.r; i += kGemvThreads) tl[i] = td[i];
      }
      __syncthreads();
    }

    // per-warp operands of the next block: X fragments and this lane's row scales
    const int ra = c0 + lane, rb = c0 + 32 + lane;
    const bool va = lane < R, vb = 32 + lane < R;
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
    // raw scale operands of block b for rows ra / rb: DQ -> (c2 byte, c2_scale), else the scale
    auto load_sc = [&](int b, uint32_t& ca, float& fa, uint32_t& cb, float& fb) {
      ca = cb = 0u;
      fa = fb = 0.0f;
      if (dq) {
        if (va) {
          const int64_t i = (int64_t)ra * nbk + b;
          ca = __ldg(p.w.c2 + i);
          fa = __ldg(p.w.c2s + (i >> 8));
        }
        if (NT > 4 && vb) {
          const int64_t i = (int64_t)rb * nbk + b;
          cb = __ldg(p.w.c2 + i);
          fb = __ldg(p.w.c2s + (i >> 8));
        }
      } else {
        if (va) fa = load_scalar(p.w.scales, p.w.sdt, (int64_t)ra * nbk + b);
        if (NT > 4 && vb) fb = load_scalar(p.w.scales, p.w.sdt, (int64_t)rb * nbk + b);
      }
    };

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    uint32_t xc[16], xn[16];
    uint32_t ca, cb, na = 0, nb2 = 0;
    float fa, fb, nfa = 0.0f, nfb = 0.0f;
    if (warp < nbk) {
      load_x(warp, xc);
      load_sc(warp, ca, fa, cb, fb);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) xc[i] = 0u;
      ca = cb = 0u;
      fa = fb = 0.0f;
    }

    for (int s = 0; s < nst; ++s) {
      const uint32_t gst = gs + s, slot = gst % S;
      if (warp == 0 && s + (int)S - 1 < nst) issue(s + (int)S - 1);
      const int b = s * kStageBlocks + warp;
      const bool active = b < nbk;
      const bool more = b + kStageBlocks < nbk;
      if (more) {
        load_x(b + kStageBlocks, xn);
        load_sc(b + kStageBlocks, na, nfa, nb2, nfb);
      }
      const float sA = dq ? sclut[ca] * fa : fa;
      const float sB = dq ? sclut[cb] * fb : fb;
      const bool ok = mbar_wait(full0 + 8 * slot, (gst / S) & 1, abortp);
      if (active && ok) {
        const unsigned char* stage = ring + slot * STAGE + warp * 32 + t * 8;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt < ntiles) {
            const uint2 cw = *reinterpret_cast<const uint2*>(stage + (nt * 8 + g) * kRowStride);
            float part[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t word = (j < 2) ? cw.x : cw.y;
              uint32_t b0, b1;
              if (j & 1) {
                b0 = lut_at<16>(word, lut_lane);
                b1 = lut_at<24>(word, lut_lane);
              } else {
                b0 = lut_at<0>(word, lut_lane);
                b1 = lut_at<8>(word, lut_lane);
              }
              if (j == 0)
                Mma16816Zero<DT>::run(part, xc[0], xc[8], xc[1], xc[9], b0, b1);
              else
                Mma16816<DT>::run(part, xc[2 * j], xc[8 + 2 * j], xc[2 * j + 1], xc[8 + 2 * j + 1], b0, b1);
            }
            const float src = nt < 4 ? sA : sB;
            const float s0 = __shfl_sync(0xffffffffu, src, (nt * 8 + 2 * t) & 31);
            const float s1 = __shfl_sync(0xffffffffu, src, (nt * 8 + 2 * t + 1) & 31);
            acc[nt][0] = fmaf(part[0], s0, acc[nt][0]);
            acc[nt][1] = fmaf(part[1], s1, acc[nt][1]);
            acc[nt][2] = fmaf(part[2], s0, acc[nt][2]);
            acc[nt][3] = fmaf(part[3], s1, acc[nt][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * slot);
      if (more) {
#pragma unroll
        for (int i = 0; i < 16; ++i) xc[i] = xn[i];
        ca = na, cb = nb2, fa = nfa, fb = nfb;
      }
    }
    gs += nst;
    if (*abortp) {
      // a wait gave up: let the copies already issued land (bounded) before
      // the ring's memory is reused or the CTA exits
      if (warp == 0)
        for (uint32_t k = 0; k < S && k < gs; ++k) {
          const uint32_t gst = gs - 1 - k, slot = gst % S;
          for (uint32_t i = 0; i < kWaitLimit; ++i) {
            uint32_t done;
            asm volatile(
                "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                : "=r"(done)
                : "r"(full0 + 8 * slot), "r"((gst / S) & 1)
                : "memory");
            if (done) break;
          }
        }
      __syncthreads();
      return;
    }

    __syncthreads();  // every warp is done reading the ring; the reduction reuses it
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      if (nt < ntiles)
        red[(warp * NT + nt) * 32 + lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
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

template <int DT, int MT, int NT>
static int nf4_launch(GemvArgs g, cudaStream_t st) {
  auto kern = gemv_nf4_k<DT, MT, NT>;
  g.stages = gemv_nf4_stages(NT, g.w.K);
  const size_t smem = gemv_nf4_smem(NT, g.w.K, g.M, g.r);
  const int rc = ensure_smem_limit((const void*)kern, smem);
  if (rc != RQ_OK) return rc;
  kern<<<g.grid, kGemvThreads, smem, st>>>(g);
  return check_launch();
}

template <int DT, int MT>
static int nf4_nt(const GemvArgs& g, int nt, cudaStream_t st) {
  switch (nt) {
    case 1: return nf4_launch<DT, MT, 1>(g, st);
    case 2: return nf4_launch<DT, MT, 2>(g, st);
    case 3: return nf4_launch<DT, MT, 3>(g, st);
    case 4: return nf4_launch<DT, MT, 4>(g, st);
    case 5: return nf4_launch<DT, MT, 5>(g, st);
    case 6: return nf4_launch<DT, MT, 6>(g, st);
    case 7: return nf4_launch<DT, MT, 7>(g, st);
    default: return nf4_launch<DT, MT, 8>(g, st);
  }
}

int gemv_nf4_launch(const GemvArgs& g, int nt, cudaStream_t st) {
  const bool m16 = g.M > 8;
  if (g.w.K % 32 || ((uintptr_t)g.w.q % 16)) return RQ_ERR_ALIGN;  // bulk copies need 16-byte rows
  if (g.xdt == RQ_BF16) return m16 ? nf4_nt<RQ_BF16, 16>(g, nt, st) : nf4_nt<RQ_BF16, 8>(g, nt, st);
  return m16 ? nf4_nt<RQ_F16, 16>(g, nt, st) : nf4_nt<RQ_F16, 8>(g, nt, st);
}

}  // namespace rq

extern "C" int rq_take_kernel_timeouts(unsigned int* count) {
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, rq::g_kernel_timeouts, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(rq::g_kernel_timeouts, &zero, sizeof(zero));
  if (e != cudaSuccess) {
    rq::set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  if (count) *count = v;
  return RQ_OK;
}
