// gemm_tcgen05.cu -- prefill/training-shaped fused NF4 dequant GEMM on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Forward  Y[M, N]  = X[M, K] . deq(W[N, K])^T (+ bias, + LoRA), and the
// transposed variant for backward  dX[M, K] = dY[M, N] . deq(W) (+ LoRA),
// for M >= 64, bf16/f16 activations, NF4 weights (plain, fp8 or int8
// double-quantized scales).
//
// CTA tile 128 (tokens) x 256 (outputs), reduction step 64.  Forward: the
// step is one quant block, so a stage needs one scale per weight row.  dX:
// the step covers 64 weight rows and the tile 256 columns (4 blocks a row);
// the dequant warps write W transposed (k-major rows of n).  One CTA per
// SM, 10 warps:
//   warp 0   TMA producer: X (dY) tile [128 x 64] per stage (128-byte
//            swizzle), and once the LoRA tiles: forward t = x.A^T [128 x r]
//            and B [256 x r] (r <= 64, zero-filled to 64 by the TMA bounds);
//            dX gt = rnd(dY*s).B [128 x r] and A [r x 256] (read as an
//            MN-major operand: four 64-column boxes);
//   warp 1   allocates 512 tensor-memory columns; lane 0 issues the MMAs:
//            tcgen05.mma kind::f16, M=128 N=256 K=16, both operands from
//            shared memory (K-major, 128-byte swizzle); the LoRA product
//            t . B^T (gt . A) goes to its own accumulator (columns 256..511)
//            so the epilogue keeps the reference's rounding sequence;
//   warps 2-9  dequantize the W tile of each stage into shared memory as
//            the reference's exact bf16/f16(T[code] * scale) values, in the
//            swizzled K-major layout the MMA reads, then run the epilogue:
//            tcgen05.ld of both accumulators (warp w reads lanes
//            32*(w%4)..., warps w and w+4 split the columns), bias and LoRA
//            rounding, Y stores.
// Stages move through mbarriers: X landed (TMA transaction bytes), W tile
// written (8 dequant-warp arrivals after a proxy fence), slot free
// (tcgen05.commit of the MMAs that read it).  Every wait is bounded; a wait
// that runs out raises the CTA's abort flag, the CTA drains its in-flight
// copies and MMAs (bounded), frees its tensor memory, skips Y and counts
// in the kernel-timeout counter.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "linear_common.cuh"
#include "rq_internal.h"

namespace rq {

// Bounded waits of this file's kernels that ran out (read and cleared with
// the GEMV's counter by rq_take_kernel_timeouts).
__device__ unsigned int g_gemm_timeouts;

// 2-D/3-D tensor map, cached (gemv_nf4.cu)
int tensor_map_encode(int type, int swz, int rank, const void* ptr, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box, CUtensorMap* out);

int gemm_take_timeouts(unsigned int* v) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(v, g_gemm_timeouts, sizeof(*v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_gemm_timeouts, &zero, sizeof(zero));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return RQ_OK;
}

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 3;
constexpr int kDqWarps = 8;                 // dequant / epilogue warps
constexpr int kThreads = 64 + kDqWarps * 32;
constexpr uint32_t kABytes = BM * BK * 2;   // 16 KB
constexpr uint32_t kBBytes = BN * BK * 2;   // 32 KB
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kTmemCols = 512;              // base accumulator 0..255, LoRA 256..511

struct GemmArgs {
  CUtensorMap xmap;   // X [M][K] (dX: dY [M][N]), box 64 x 128, 128-byte swizzle
  CUtensorMap tmap;   // t [M][r] (dX: gt), box 64 x 128, 128-byte swizzle (r < 64 zero-filled)
  CUtensorMap bmap;   // LoRA B [N][r], box 64 x 256 (dX: A [r][K], box 64 x 64), 128-byte swizzle
  QWeight w;
  const void* bias;
  int bdt;
  void* y;            // Y [M][N] (dX: dX [M][K])
  int M, N, K, r;
  float s;            // LoRA scaling (dX: 1, gt already carries it)
};

// dynamic shared memory layout (1 KB aligned base)
constexpr uint32_t kSmA = 0;                               // kStages x 16 KB
constexpr uint32_t kSmB = kSmA + kStages * kABytes;        // kStages x 32 KB
constexpr uint32_t kSmT = kSmB + kStages * kBBytes;        // LoRA t tile, 16 KB
constexpr uint32_t kSmLB = kSmT + kABytes;                 // LoRA B tile, 32 KB
constexpr int kLutReps = 16;                               // copies of the code-byte table (one per half-warp lane)
constexpr uint32_t kSmLut = kSmLB + kBBytes;               // code byte -> (T[lo], T[hi]), 8 copies interleaved
constexpr uint32_t kSmScl = kSmLut + 256 * kLutReps * 8;   // 256 fp32 second-level values
constexpr uint32_t kSmBytes = kSmScl + 256 * 4 + 1024;     // + alignment slack

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_test(bar, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1;
  atomicAdd(&g_gemm_timeouts, 1u);
  return false;
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory descriptor of a K-major operand tile with 128-byte swizzle:
// rows of 128 bytes (64 16-bit elements), 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                         // layout: 128-byte swizzle
  return d;
}

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle:
// rows (K) of 128 bytes = 64 MN elements, 8-row groups 1024 bytes apart,
// 64-element MN groups `lbo` bytes apart.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: 16-bit A/B of type DT, fp32 accumulate, A K-major,
// B K-major (or MN-major), M=128, N=256.
template <int DT>
__device__ __forceinline__ uint32_t idesc_f16(bool b_mn = false) {
  const uint32_t ab = DT == RQ_BF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive fp32 columns of this thread's accumulator row
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// two fp32 values rounded to the 16-bit type DT (one packed convert)
template <int DT>
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  if constexpr (DT == RQ_BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <int DT, bool DX>
__global__ void __launch_bounds__(kThreads, 1) gemm_k(const __grid_constant__ GemmArgs g) {
  using T = typename DType<DT>::T;
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t bars[3 * kStages + 3];  // fullA[S], fullB[S], empty[S], lora, acc, drain
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag, a_issued, mma_done;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1 KB aligned view of the dynamic shared memory (swizzle atoms)
  const uint32_t sraw = smem_u32(dsm);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  unsigned char* sm = dsm + (sbase - sraw);
  const uint32_t fullA0 = smem_u32(bars), fullB0 = fullA0 + 8 * kStages, empty0 = fullB0 + 8 * kStages;
  const uint32_t lorabar = empty0 + 8 * kStages, accbar = lorabar + 8, drainbar = accbar + 8;
  volatile int* abortp = &abort_flag;

  const int M = g.M, N = g.N, K = g.K;
  const int W_out = DX ? K : N;  // output columns
  const int nkb = (DX ? N : K) / BK;  // reduction steps
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const bool has_lora = g.r > 0;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(fullA0 + 8 * i, 1);
      mbar_init(fullB0 + 8 * i, kDqWarps);
      mbar_init(empty0 + 8 * i, 1);
    }
    mbar_init(lorabar, 1);
    mbar_init(accbar, 1);
    mbar_init(drainbar, 1);
    abort_flag = 0;
    a_issued = 0;
    mma_done = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // whole warp: tensor-memory allocation
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // code byte v -> (T[v & 15], T[v >> 4]) in kLutReps interleaved copies
  // (entry v, copy c at (v * kLutReps + c) * 8: lane l reads copy l % 16, so
  // the 16 lanes of a half warp hit 16 distinct bank pairs), and the
  // second-level table
  float2* lutp = reinterpret_cast<float2*>(sm + kSmLut);
  float* sclut = reinterpret_cast<float*>(sm + kSmScl);
  for (int i = tid; i < 256 * kLutReps; i += kThreads) {
    const int v = i / kLutReps;
    lutp[i] = make_float2(kNF4[v & 15], kNF4[v >> 4]);
  }
  if (g.w.fmt != RQ_W_NF4)
    for (int v = tid; v < 256; v += kThreads)
      sclut[v] = g.w.fmt == RQ_W_NF4_DQ_FP8 ? e4m3fnuz_to_f32(v) : ieee_div((float)(int8_t)v, 127.0f);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      if (has_lora) {
        mbar_expect_tx(lorabar, kABytes + kBBytes);
        tma_2d(sbase + kSmT, &g.tmap, 0, m0, lorabar);
        if (DX) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_2d(sbase + kSmLB + j * 8192, &g.bmap, n0 + 64 * j, 0, lorabar);
        } else {
          tma_2d(sbase + kSmLB, &g.bmap, 0, n0, lorabar);
        }
      }
      for (int kb = 0; kb < nkb; ++kb) {
        const int slot = kb % kStages;
        if (kb >= kStages && !mbar_wait(empty0 + 8 * slot, ((kb / kStages) - 1) & 1, abortp)) break;
        mbar_expect_tx(fullA0 + 8 * slot, kABytes);
        tma_2d(sbase + kSmA + slot * kABytes, &g.xmap, kb * BK, m0, fullA0 + 8 * slot);
        *reinterpret_cast<volatile int*>(&a_issued) = kb + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<DT>();
      bool ok = true;
      if (has_lora) {
        ok = mbar_wait(lorabar, 0, abortp);
        if (ok) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t db = DX ? sw128_mn_desc(sbase + kSmLB + kk * 2048, 8192)  // rows 16kk.. of A
                                   : sw128_desc(sbase + kSmLB + kk * 32);
            mma_f16(tmem + 256, sw128_desc(sbase + kSmT + kk * 32), db, DX ? idesc_f16<DT>(true) : idesc, kk > 0);
          }
        }
      }
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int slot = kb % kStages;
        const uint32_t par = (kb / kStages) & 1;
        if (!mbar_wait(fullA0 + 8 * slot, par, abortp) || !mbar_wait(fullB0 + 8 * slot, par, abortp)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a = sbase + kSmA + slot * kABytes, b = sbase + kSmB + slot * kBBytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_f16(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(empty0 + 8 * slot);  // the slot is free once these MMAs have read it
        *reinterpret_cast<volatile int*>(&mma_done) = kb + 1;
      }
      mma_commit(accbar);  // every MMA issued so far is complete
    }
  } else {
    // ------------------------------------------------ dequant warps (2..9)
    // Thread dt owns, per stage: forward tile row dt (weight row n0 + dt,
    // block kb); dX the 32 codes [32 hf, 32 hf + 32) of block n0/64 + qb4 of
    // weight rows 64 kb + 2p and +1 (p = dt % 32, qb4 = dt / 64, hf = dt / 32
    // % 2: a warp's 32 lanes then write one shared row's 32 distinct words).
    // Raw codes and scales are loaded two stages ahead.
    const int dt = tid - 64;
    const int fmt = g.w.fmt;
    const int nbk = K / 64;
    const uint8_t* qb = static_cast<const uint8_t*>(g.w.q);
    const int p = dt & 31, qb4 = dt >> 6, hf = (dt >> 5) & 1;
    const uint32_t lut_lane = smem_u32(lutp) + (uint32_t)(lane & (kLutReps - 1)) * 8;
    // (T[lo], T[hi]) of byte J of `w`: one byte permute, one multiply-add, one 8-byte load
    auto lut_at = [&](uint32_t w, int j) -> float2 {
      const uint32_t addr = __byte_perm(w, 0u, 0x4440u | (uint32_t)j) * (kLutReps * 8) + lut_lane;
      float2 v;
      asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
      return v;
    };
    struct Raw {
      uint4 c[2];  // forward: 32 code bytes of the row; dX: 16 bytes of each of the two rows
      uint32_t c2b[2];
      float sraw[2];
    };
    auto fetch = [&](int kb, Raw& r) {
      r.c[0] = r.c[1] = make_uint4(0u, 0u, 0u, 0u);
      r.c2b[0] = r.c2b[1] = 0u;
      r.sraw[0] = r.sraw[1] = 0.0f;
      if (kb >= nkb) return;
#pragma unroll
      for (int h = 0; h < (DX ? 2 : 1); ++h) {
        const int n = DX ? kb * 64 + 2 * p + h : n0 + dt;
        const int blk = DX ? (n0 >> 6) + qb4 : kb;
        if (DX ? blk < nbk : n < N) {
          const uint4* src = reinterpret_cast<const uint4*>(qb + (size_t)n * (K / 2) + (size_t)blk * 32);
          if (DX) {
            r.c[h] = __ldg(src + hf);
          } else {
            r.c[0] = __ldg(src);
            r.c[1] = __ldg(src + 1);
          }
          const int64_t bi = (int64_t)n * nbk + blk;
          if (fmt == RQ_W_NF4) {
            r.sraw[h] = load_scalar(g.w.scales, g.w.sdt, bi);
          } else {
            r.c2b[h] = __ldg(g.w.c2 + bi);
            r.sraw[h] = __ldg(g.w.c2s + bi / kDQBlock2);
          }
        }
      }
    };
    auto convert = [&](int kb, const Raw& r) -> bool {
      const int slot = kb % kStages;
      float sv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) sv[h] = fmt == RQ_W_NF4 ? r.sraw[h] : sclut[r.c2b[h]] * r.sraw[h];
      if (kb >= kStages && !mbar_wait(empty0 + 8 * slot, ((kb / kStages) - 1) & 1, abortp)) return false;
      unsigned char* bt = sm + kSmB + slot * kBBytes;
      if (DX) {
        // tile row k (= output column), 16-bit pair (n, n+1) at column 2p
        const uint32_t colb = (uint32_t)(p >> 2), colo = (uint32_t)(p & 3) * 4;
        const uint32_t w0[4] = {r.c[0].x, r.c[0].y, r.c[0].z, r.c[0].w};
        const uint32_t w1[4] = {r.c[1].x, r.c[1].y, r.c[1].z, r.c[1].w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 l0 = lut_at(w0[i], j), l1 = lut_at(w1[i], j);
            const int kr = qb4 * 64 + hf * 32 + i * 8 + j * 2;  // tile rows kr (low nibbles), kr + 1 (high)
            unsigned char* r0 = bt + (kr >> 3) * 1024 + (kr & 7) * 128 + colo;
            unsigned char* r1 = bt + ((kr + 1) >> 3) * 1024 + ((kr + 1) & 7) * 128 + colo;
            *reinterpret_cast<uint32_t*>(r0 + ((colb ^ (kr & 7)) << 4)) = pack_rn<DT>(l0.x * sv[0], l1.x * sv[1]);
            *reinterpret_cast<uint32_t*>(r1 + ((colb ^ ((kr + 1) & 7)) << 4)) = pack_rn<DT>(l0.y * sv[0], l1.y * sv[1]);
          }
      } else {
        // 8 chunks of 16 bytes (8 elements) a row; chunk c at (c ^ (row & 7))
        const uint32_t cw[8] = {r.c[0].x, r.c[0].y, r.c[0].z, r.c[0].w, r.c[1].x, r.c[1].y, r.c[1].z, r.c[1].w};
        unsigned char* rowp = bt + (dt >> 3) * 1024 + (dt & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t qv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 l = lut_at(cw[c], j);
            qv[j] = pack_rn<DT>(l.x * sv[0], l.y * sv[0]);
          }
          *reinterpret_cast<uint4*>(rowp + ((c ^ (dt & 7)) << 4)) = make_uint4(qv[0], qv[1], qv[2], qv[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive(fullB0 + 8 * slot);
      return true;
    };
    Raw ra, rb;
    fetch(0, ra);
    fetch(1, rb);
    for (int kb = 0; kb < nkb; kb += 2) {
      if (!convert(kb, ra)) break;
      fetch(kb + 2, ra);
      if (kb + 1 >= nkb) break;
      if (!convert(kb + 1, rb)) break;
      fetch(kb + 3, rb);
    }

    // ---------------------------------------------------------- epilogue
    const bool ok = mbar_wait(accbar, 0, abortp) && !*abortp;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int quad = warp & 3;  // tensor-memory lanes 32*quad ... are this warp's rows
    const int row = quad * 32 + lane, m = m0 + row;
    const int c_lo = ((warp - 2) >> 2) * (BN / 2);  // warps w and w+4 split the columns
    const bool has_bias = !DX && g.bias != nullptr;
    T* y = static_cast<T*>(g.y);
    for (int cb = c_lo; cb < c_lo + BN / 2; cb += 32) {
      float acc[32], u[32];
      tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + cb, acc);
      if (has_lora) tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + 256 + cb, u);
      if (!ok || m >= M) continue;
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float o[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int n = n0 + cb + j + e;
          const float bv = (has_bias && n < W_out) ? load_scalar(g.bias, g.bdt, n) : 0.0f;
          o[e] = lora_epilogue<DT>(acc[j + e], has_bias, bv, has_lora ? u[j + e] : 0.0f, has_lora, g.s);
        }
        pk[j / 2] = pack_rn<DT>(o[0], o[1]);
      }
      T* yrow = y + (size_t)m * W_out + n0 + cb;
      if (n0 + cb + 32 <= W_out && ((reinterpret_cast<uintptr_t>(yrow) & 15) == 0)) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          reinterpret_cast<uint4*>(yrow)[q4] = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
      } else {
        for (int j = 0; j < 32 && n0 + cb + j < W_out; ++j) {
          const uint32_t w2 = pk[j / 2];
          const uint16_t hbits = (j & 1) ? (uint16_t)(w2 >> 16) : (uint16_t)(w2 & 0xFFFF);
          reinterpret_cast<uint16_t*>(yrow)[j] = hbits;
        }
      }
    }
  }

  // ---------------------------------------------------------- teardown
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    if (*abortp && lane == 0) {
      // MMAs may still be in flight: wait (bounded) for all of them, and for
      // the TMA copies the producer issued but no MMA waited for, before
      // the tensor and shared memory are released
      mma_commit(drainbar);
      for (uint32_t i = 0; i < kWaitLimit && !mbar_test(drainbar, 0); ++i) {
      }
      const int done = *reinterpret_cast<volatile int*>(&mma_done), issued = *reinterpret_cast<volatile int*>(&a_issued);
      for (int kb = done; kb < issued; ++kb)
        for (uint32_t i = 0; i < kWaitLimit && !mbar_test(fullA0 + 8 * (kb % kStages), (kb / kStages) & 1); ++i) {
        }
      if (has_lora)
        for (uint32_t i = 0; i < kWaitLimit && !mbar_test(lorabar, 0); ++i) {
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

// ---------------------------------------------------------------- host side

bool gemm_supported(const LinearArgs& a, bool dx) {
  if (a.M < 64 || !is_nf4_fmt(a.w.fmt) || a.w.bs != 64 || a.w.K % 64) return false;
  if (dx && a.w.N % 64) return false;  // dX reduces over N in steps of 64 rows
  if (a.xdt != RQ_BF16 && a.xdt != RQ_F16) return false;
  if (a.r > 64 || (a.r > 0 && a.r % 8)) return false;
  if ((uintptr_t)a.x % 16 || (uintptr_t)a.w.q % 16) return false;
  if (a.r > 0 && (uintptr_t)a.lora_b % 16) return false;
  return a.w.N <= 0x7fffffff && a.w.K <= 0x7fffffff && a.M <= 0x7fffffff;
}

// Shared launch of both variants: `a_op` is X (forward) or dY (dX), `t` the
// down product (t or gt), `bmat` LoRA B (forward) or A (dX).
static int gemm_launch(const LinearArgs& a, bool dx, const void* a_op, const void* t, cudaStream_t st) {
  GemmArgs g;
  const uint64_t M = (uint64_t)a.M, N = (uint64_t)a.w.N, K = (uint64_t)a.w.K, r = (uint64_t)(a.r > 0 ? a.r : 8);
  const uint64_t red = dx ? N : K, wout = dx ? K : N;
  const int ty = CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const int swz = CU_TENSOR_MAP_SWIZZLE_128B;
  {
    const uint64_t d[3] = {red, M, 1}, s[2] = {red * 2, 0};
    const uint32_t b[3] = {BK, BM, 1};
    const int rc = tensor_map_encode(ty, swz, 2, a_op, d, s, b, &g.xmap);
    if (rc != RQ_OK) return rc;
  }
  if (a.r > 0) {
    const uint64_t dt[3] = {r, M, 1}, st2[2] = {r * 2, 0};
    const uint32_t bt[3] = {BK, BM, 1};
    int rc = tensor_map_encode(ty, swz, 2, t, dt, st2, bt, &g.tmap);
    if (rc != RQ_OK) return rc;
    if (dx) {  // A [r][K]: 64 columns x 64 rows a box (rows past r zero-filled)
      const uint64_t db[3] = {K, r, 1}, sb[2] = {K * 2, 0};
      const uint32_t bb[3] = {64, 64, 1};
      rc = tensor_map_encode(ty, swz, 2, a.lora_a, db, sb, bb, &g.bmap);
    } else {  // B [N][r]
      const uint64_t db[3] = {r, N, 1}, sb[2] = {r * 2, 0};
      const uint32_t bb[3] = {BK, BN, 1};
      rc = tensor_map_encode(ty, swz, 2, a.lora_b, db, sb, bb, &g.bmap);
    }
    if (rc != RQ_OK) return rc;
  } else {
    g.tmap = g.xmap;
    g.bmap = g.xmap;
  }
  g.w = a.w;
  g.bias = dx ? nullptr : a.bias;
  g.bdt = a.bdt;
  g.y = a.y;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.r = a.r > 0 ? a.r : 0;
  g.s = dx ? 1.0f : a.scaling;
  const dim3 grid((unsigned)((wout + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  const void* kern = a.xdt == RQ_BF16 ? (dx ? (const void*)gemm_k<RQ_BF16, true> : (const void*)gemm_k<RQ_BF16, false>)
                                      : (dx ? (const void*)gemm_k<RQ_F16, true> : (const void*)gemm_k<RQ_F16, false>);
  const int rc = ensure_smem_limit(kern, kSmBytes);
  if (rc != RQ_OK) return rc;
  if (a.xdt == RQ_BF16) {
    if (dx)
      gemm_k<RQ_BF16, true><<<grid, kThreads, kSmBytes, st>>>(g);
    else
      gemm_k<RQ_BF16, false><<<grid, kThreads, kSmBytes, st>>>(g);
  } else {
    if (dx)
      gemm_k<RQ_F16, true><<<grid, kThreads, kSmBytes, st>>>(g);
    else
      gemm_k<RQ_F16, false><<<grid, kThreads, kSmBytes, st>>>(g);
  }
  return check_launch();
}

int gemm_forward(const LinearArgs& a, const void* tdown, cudaStream_t st) { return gemm_launch(a, false, a.x, tdown, st); }

// dX: a.x is dY [M][N], gt = rnd(rnd(dY*s).B) [M][r], a.y the dX output.
int gemm_dx(const LinearArgs& a, const void* gt, cudaStream_t st) {
  if (a.r > 0 && ((uintptr_t)a.lora_a % 16 || (a.w.K * 2) % 16)) return RQ_ERR_ALIGN;
  return gemm_launch(a, true, a.x, gt, st);
}

}  // namespace rq
