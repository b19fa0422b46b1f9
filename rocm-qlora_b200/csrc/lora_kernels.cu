// lora_kernels.cu -- the rank-r "down" products of the LoRA adapter.
//
//   forward: t[M, r]  = rnd(x[M, K] . A[r, K]^T)            (lora_layer.py:67, x @ A.T)
//   dx:      gt[M, r] = rnd(rnd(dy[M, N] * s) . B[N, r])     (autograd of (.. @ B.T) * s)
//
// Both are skinny GEMMs (r <= 128).  They run on the tensor cores with
// mma.sync m16n8k16 (fp32 accumulation); when M is small the reduction
// dimension is split across CTAs and the fp32 partials are summed in a
// fixed order by the last CTA to finish (arrival counter in the workspace
// counter area, reset by that CTA), so results are deterministic.
#include <cuda_runtime.h>

#include "linear_common.cuh"

namespace rq {

template <int DT> struct MmaOp;
template <> struct MmaOp<RQ_BF16> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct MmaOp<RQ_F16> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <int DT>
__device__ __forceinline__ uint16_t bits16(typename DType<DT>::T v) {
  return *reinterpret_cast<uint16_t*>(&v);
}

// Two consecutive 16-bit elements p[i], p[i+1] (zero past `lim`).
template <int DT>
__device__ __forceinline__ uint32_t ld_pair(const typename DType<DT>::T* p, int64_t i, int64_t lim, bool vec_ok) {
  if (vec_ok && i + 1 < lim) return *reinterpret_cast<const uint32_t*>(p + i);
  const uint32_t lo = i < lim ? bits16<DT>(p[i]) : 0u;
  const uint32_t hi = i + 1 < lim ? bits16<DT>(p[i + 1]) : 0u;
  return lo | (hi << 16);
}

template <int DT>
__device__ __forceinline__ uint32_t prescale_pair(uint32_t v, float s) {
  using T = typename DType<DT>::T;
  const uint16_t lo = (uint16_t)(v & 0xFFFFu), hi = (uint16_t)(v >> 16);
  const float a = DType<DT>::to_f32(*reinterpret_cast<const T*>(&lo)) * s;
  const float b = DType<DT>::to_f32(*reinterpret_cast<const T*>(&hi)) * s;
  return pack2<DT>(a, b);
}

constexpr int kLoraMaxR = 128;

// out[M, R] = rnd(pre(X)[M, Kr] . W2^T);  W2 is [R, Kr] (WT = false) or
// [Kr, R] (WT = true).  grid = (ceil(M / (16*WM)), ksplit).
template <int DT, bool WT, int WM>
__global__ void __launch_bounds__(32 * WM) lora_down_mma_k(const typename DType<DT>::T* __restrict__ X, int64_t M,
                                                           int64_t Kr, const typename DType<DT>::T* __restrict__ W2,
                                                           int R, float pre_s, int do_pre, int kchunk,
                                                           float* __restrict__ partial, unsigned* __restrict__ counters,
                                                           typename DType<DT>::T* __restrict__ out) {
  using T = typename DType<DT>::T;
  constexpr int NT = kLoraMaxR / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t m0 = ((int64_t)blockIdx.x * WM + warp) * 16;
  const int64_t kbeg = (int64_t)blockIdx.y * kchunk;
  const int64_t kend = kbeg + kchunk < Kr ? kbeg + kchunk : Kr;
  const int ntiles = (R + 7) / 8;
  const bool vec_x = ((uintptr_t)X % 4 == 0) && (Kr % 2 == 0);
  const bool vec_w = ((uintptr_t)W2 % 4 == 0) && (Kr % 2 == 0);
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

  const int64_t ra = m0 + g, rb = m0 + g + 8;
  const T* xa = X + (ra < M ? ra : 0) * Kr;
  const T* xb = X + (rb < M ? rb : 0) * Kr;
  for (int64_t k0 = kbeg; k0 < kend; k0 += 16) {
    uint32_t a[4];
    a[0] = ra < M ? ld_pair<DT>(xa, k0 + 2 * t, kend, vec_x) : 0u;
    a[1] = rb < M ? ld_pair<DT>(xb, k0 + 2 * t, kend, vec_x) : 0u;
    a[2] = ra < M ? ld_pair<DT>(xa, k0 + 8 + 2 * t, kend, vec_x) : 0u;
    a[3] = rb < M ? ld_pair<DT>(xb, k0 + 8 + 2 * t, kend, vec_x) : 0u;
    if (do_pre) {
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = prescale_pair<DT>(a[i], pre_s);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt < ntiles) {
        const int n = nt * 8 + g;
        uint32_t b0 = 0, b1 = 0;
        if (n < R) {
          if (!WT) {
            b0 = ld_pair<DT>(W2 + (int64_t)n * Kr, k0 + 2 * t, kend, vec_w);
            b1 = ld_pair<DT>(W2 + (int64_t)n * Kr, k0 + 8 + 2 * t, kend, vec_w);
          } else {
            const int64_t ka = k0 + 2 * t, kb = k0 + 8 + 2 * t;
            const uint32_t e0 = ka < kend ? bits16<DT>(W2[ka * R + n]) : 0u;
            const uint32_t e1 = ka + 1 < kend ? bits16<DT>(W2[(ka + 1) * R + n]) : 0u;
            const uint32_t e2 = kb < kend ? bits16<DT>(W2[kb * R + n]) : 0u;
            const uint32_t e3 = kb + 1 < kend ? bits16<DT>(W2[(kb + 1) * R + n]) : 0u;
            b0 = e0 | (e1 << 16);
            b1 = e2 | (e3 << 16);
          }
        }
        MmaOp<DT>::mma(acc[nt], a, b0, b1);
      }
    }
  }

  if (gridDim.y == 1) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt < ntiles) {
        const int c = nt * 8 + 2 * t;
        if (ra < M && c < R) out[ra * R + c] = DType<DT>::from_f32(acc[nt][0]);
        if (ra < M && c + 1 < R) out[ra * R + c + 1] = DType<DT>::from_f32(acc[nt][1]);
        if (rb < M && c < R) out[rb * R + c] = DType<DT>::from_f32(acc[nt][2]);
        if (rb < M && c + 1 < R) out[rb * R + c + 1] = DType<DT>::from_f32(acc[nt][3]);
      }
    }
    return;
  }
  // split-K: partial[split][m][c] fp32, the last CTA of this M-tile sums
  float* mypart = partial + (int64_t)blockIdx.y * M * R;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    if (nt < ntiles) {
      const int c = nt * 8 + 2 * t;
      if (ra < M && c < R) mypart[ra * R + c] = acc[nt][0];
      if (ra < M && c + 1 < R) mypart[ra * R + c + 1] = acc[nt][1];
      if (rb < M && c < R) mypart[rb * R + c] = acc[nt][2];
      if (rb < M && c + 1 < R) mypart[rb * R + c + 1] = acc[nt][3];
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ unsigned ticket;
  if (threadIdx.x == 0) ticket = atomicAdd(&counters[blockIdx.x], 1u);
  __syncthreads();
  if (ticket != gridDim.y - 1) return;
  __threadfence();
  const int64_t mt0 = (int64_t)blockIdx.x * WM * 16;
  const int64_t mt1 = mt0 + WM * 16 < M ? mt0 + WM * 16 : M;
  for (int64_t i = threadIdx.x; i < (mt1 - mt0) * R; i += blockDim.x) {
    const int64_t m = mt0 + i / R, c = i % R;
    float s = 0.0f;
    for (unsigned sp = 0; sp < gridDim.y; ++sp) s += __ldcg(&partial[(int64_t)sp * M * R + m * R + c]);
    out[m * R + c] = DType<DT>::from_f32(s);
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;  // leave the counter area zeroed
}

// Small M (<= 16): a cluster of kLoraCluster CTAs x 16 warps splits the
// reduction dimension; each CTA reduces its warps in shared memory, then
// every CTA sums its share of the outputs over the cluster's partials
// through distributed shared memory, in rank order (deterministic).  A warp
// issues the loads of KB k-steps before their MMAs.  NT = r/8 rounded up
// to 2, 4 or 8 (r <= 64).
constexpr int kLoraCluster = 8;
constexpr int kLoraSmallMaxR = 64;
constexpr int kLoraSmallWarps = 16;

template <int DT, bool WT, int NT>
__global__ void __cluster_dims__(kLoraCluster, 1, 1) __launch_bounds__(kLoraSmallWarps * 32)
    lora_down_small_k(const typename DType<DT>::T* __restrict__ X, int M, int Kr,
                      const typename DType<DT>::T* __restrict__ W2, int R, float pre_s, int do_pre,
                      typename DType<DT>::T* __restrict__ out) {
  using T = typename DType<DT>::T;
  // Launched as the programmatic dependent of the kernel before it in the
  // stream (it may be resident before that kernel ends): wait until that
  // kernel has finished and its writes are visible (X may be its output),
  // and only then let the layer's GEMV launch, which reads X at once and
  // `out` only after this grid ends.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  constexpr int RP = NT * 8;            // padded output columns
  constexpr int KB = NT <= 4 ? 8 : 4;   // k-steps per load batch
  extern __shared__ float lsm[];
  float* part = lsm;                              // [warps][16][RP]
  float* cta = lsm + kLoraSmallWarps * 16 * RP;   // [16][RP]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const unsigned rank = blockIdx.x % kLoraCluster;
  const int ksteps = (Kr + 15) / 16;
  const int nw = kLoraSmallWarps * kLoraCluster;
  const int gw = rank * kLoraSmallWarps + warp;
  const int s0 = ksteps * gw / nw, s1 = ksteps * (gw + 1) / nw;
  const bool vec_x = ((uintptr_t)X % 4 == 0) && (Kr % 2 == 0);
  const bool vec_w = ((uintptr_t)W2 % 4 == 0) && (Kr % 2 == 0);
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  const T* xa = X + (size_t)(g < M ? g : 0) * Kr;
  const T* xb = X + (size_t)(g + 8 < M ? g + 8 : 0) * Kr;
  for (int sb = s0; sb < s1; sb += KB) {
    uint32_t a[KB][4];
    uint32_t bw[KB][NT][2];
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      const int k0 = (sb + q) * 16;
      const bool on = sb + q < s1;
      a[q][0] = on && g < M ? ld_pair<DT>(xa, k0 + 2 * t, Kr, vec_x) : 0u;
      a[q][1] = on && g + 8 < M ? ld_pair<DT>(xb, k0 + 2 * t, Kr, vec_x) : 0u;
      a[q][2] = on && g < M ? ld_pair<DT>(xa, k0 + 8 + 2 * t, Kr, vec_x) : 0u;
      a[q][3] = on && g + 8 < M ? ld_pair<DT>(xb, k0 + 8 + 2 * t, Kr, vec_x) : 0u;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + g;
        uint32_t b0 = 0, b1 = 0;
        if (on && n < R) {
          if (!WT) {
            b0 = ld_pair<DT>(W2 + (size_t)n * Kr, k0 + 2 * t, Kr, vec_w);
            b1 = ld_pair<DT>(W2 + (size_t)n * Kr, k0 + 8 + 2 * t, Kr, vec_w);
          } else {
            const int ka = k0 + 2 * t, kb = k0 + 8 + 2 * t;
            const uint32_t e0 = ka < Kr ? bits16<DT>(W2[(size_t)ka * R + n]) : 0u;
            const uint32_t e1 = ka + 1 < Kr ? bits16<DT>(W2[(size_t)(ka + 1) * R + n]) : 0u;
            const uint32_t e2 = kb < Kr ? bits16<DT>(W2[(size_t)kb * R + n]) : 0u;
            const uint32_t e3 = kb + 1 < Kr ? bits16<DT>(W2[(size_t)(kb + 1) * R + n]) : 0u;
            b0 = e0 | (e1 << 16);
            b1 = e2 | (e3 << 16);
          }
        }
        bw[q][nt][0] = b0;
        bw[q][nt][1] = b1;
      }
    }
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      if (do_pre) {
#pragma unroll
        for (int i = 0; i < 4; ++i) a[q][i] = prescale_pair<DT>(a[q][i], pre_s);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) MmaOp<DT>::mma(acc[nt], a[q], bw[q][nt][0], bw[q][nt][1]);
    }
  }
  float* mine = part + warp * 16 * RP;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int c = nt * 8 + 2 * t;
    mine[g * RP + c] = acc[nt][0];
    mine[g * RP + c + 1] = acc[nt][1];
    mine[(g + 8) * RP + c] = acc[nt][2];
    mine[(g + 8) * RP + c + 1] = acc[nt][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * RP; i += blockDim.x) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kLoraSmallWarps; ++w) v += part[w * 16 * RP + i];
    cta[i] = v;
  }
  // every CTA of the cluster has its partial in shared memory
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
  const int total = M * R;
  const int share = (total + kLoraCluster - 1) / kLoraCluster;
  const uint32_t cta_addr = (uint32_t)__cvta_generic_to_shared(cta);
  for (int o = rank * share + threadIdx.x; o < total && o < (int)(rank + 1) * share; o += blockDim.x) {
    const int m = o / R, c = o % R;
    const uint32_t off = (uint32_t)(m * RP + c) * 4;
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < kLoraCluster; ++q) {
      uint32_t remote;
      float v;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(cta_addr + off), "r"(q));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote));
      sum += v;
    }
    out[(size_t)m * R + c] = DType<DT>::from_f32(sum);
  }
  // keep this CTA's shared memory alive until the cluster has read it
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

template <int DT, bool WT, int NT>
static int lora_small_launch(const void* X, int M, int Kr, const void* W2, int R, float pre_s, int do_pre, void* out,
                             cudaStream_t st) {
  using T = typename DType<DT>::T;
  const size_t smem = (size_t)(kLoraSmallWarps + 1) * 16 * NT * 8 * sizeof(float);
  auto kern = lora_down_small_k<DT, WT, NT>;
  const int rc = ensure_smem_limit((const void*)kern, smem);
  if (rc != RQ_OK) return rc;
  // programmatic dependent of the kernel before it (see the kernel's first lines)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kLoraCluster);
  cfg.blockDim = dim3(kLoraSmallWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (T*)out);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return check_launch();
}

// fp32 activations: one thread per output, CUDA cores.
// M > 16: one CTA of kWideWarps warps per 16 rows of X.  The warps split
// the reduction dimension into contiguous chunks (16-aligned), each
// loading the next k-step's fragments while it multiplies the current one,
// and meet in shared memory in a fixed order (deterministic, no workspace).
constexpr int kWideWarps = 8;

template <int DT, bool WT, int NT>
__global__ void __launch_bounds__(kWideWarps * 32) lora_down_wide_k(const typename DType<DT>::T* __restrict__ X,
                                                                     int64_t M, int64_t Kr,
                                                                     const typename DType<DT>::T* __restrict__ W2,
                                                                     int R, float pre_s, int do_pre,
                                                                     typename DType<DT>::T* __restrict__ out) {
  using T = typename DType<DT>::T;
  constexpr int RP = NT * 8 + 4;  // padded row of the partials
  __shared__ float part[kWideWarps][16][RP];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t m0 = (int64_t)blockIdx.x * 16;
  const int64_t steps = (Kr + 15) / 16;
  const int64_t s0 = steps * warp / kWideWarps, s1 = steps * (warp + 1) / kWideWarps;
  const bool vec_x = ((uintptr_t)X % 4 == 0) && (Kr % 2 == 0);
  const bool vec_w = ((uintptr_t)W2 % 4 == 0) && (Kr % 2 == 0);
  const int64_t ra = m0 + g, rb = m0 + g + 8;
  const T* xa = X + (ra < M ? ra : 0) * Kr;
  const T* xb = X + (rb < M ? rb : 0) * Kr;
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  auto load = [&](int64_t st, uint32_t (&a)[4], uint32_t (&b)[NT][2]) {
    const int64_t k0 = st * 16;
    a[0] = ra < M ? ld_pair<DT>(xa, k0 + 2 * t, Kr, vec_x) : 0u;
    a[1] = rb < M ? ld_pair<DT>(xb, k0 + 2 * t, Kr, vec_x) : 0u;
    a[2] = ra < M ? ld_pair<DT>(xa, k0 + 8 + 2 * t, Kr, vec_x) : 0u;
    a[3] = rb < M ? ld_pair<DT>(xb, k0 + 8 + 2 * t, Kr, vec_x) : 0u;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
      uint32_t b0 = 0, b1 = 0;
      if (n < R) {
        if (!WT) {
          b0 = ld_pair<DT>(W2 + (int64_t)n * Kr, k0 + 2 * t, Kr, vec_w);
          b1 = ld_pair<DT>(W2 + (int64_t)n * Kr, k0 + 8 + 2 * t, Kr, vec_w);
        } else {
          const int64_t ka = k0 + 2 * t, kb = k0 + 8 + 2 * t;
          const uint32_t e0 = ka < Kr ? bits16<DT>(W2[ka * R + n]) : 0u;
          const uint32_t e1 = ka + 1 < Kr ? bits16<DT>(W2[(ka + 1) * R + n]) : 0u;
          const uint32_t e2 = kb < Kr ? bits16<DT>(W2[kb * R + n]) : 0u;
          const uint32_t e3 = kb + 1 < Kr ? bits16<DT>(W2[(kb + 1) * R + n]) : 0u;
          b0 = e0 | (e1 << 16);
          b1 = e2 | (e3 << 16);
        }
      }
      b[nt][0] = b0;
      b[nt][1] = b1;
    }
  };
  uint32_t a[2][4], b[2][NT][2];
  if (s0 < s1) load(s0, a[0], b[0]);
  for (int64_t st = s0; st < s1; st += 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (st + h < s1) {
        if (st + h + 1 < s1) load(st + h + 1, a[h ^ 1], b[h ^ 1]);
        uint32_t av[4] = {a[h][0], a[h][1], a[h][2], a[h][3]};
        if (do_pre) {
#pragma unroll
          for (int i = 0; i < 4; ++i) av[i] = prescale_pair<DT>(av[i], pre_s);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) MmaOp<DT>::mma(acc[nt], av, b[h][nt][0], b[h][nt][1]);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int c = nt * 8 + 2 * t;
    part[warp][g][c] = acc[nt][0];
    part[warp][g][c + 1] = acc[nt][1];
    part[warp][g + 8][c] = acc[nt][2];
    part[warp][g + 8][c + 1] = acc[nt][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * R; i += blockDim.x) {
    const int rr = i / R, c = i - rr * R;
    const int64_t m = m0 + rr;
    if (m >= M) continue;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWideWarps; ++w) v += part[w][rr][c];
    out[m * R + c] = DType<DT>::from_f32(v);
  }
}

template <bool WT>
__global__ void __launch_bounds__(256) lora_down_f32_k(const float* __restrict__ X, int64_t M, int64_t Kr,
                                                       const float* __restrict__ W2, int R, float pre_s, int do_pre,
                                                       float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * R) return;
  const int64_t m = i / R, c = i % R;
  float acc = 0.0f;
  for (int64_t k = 0; k < Kr; ++k) {
    float xv = X[m * Kr + k];
    if (do_pre) xv = xv * pre_s;
    const float wv = WT ? W2[k * R + c] : W2[c * Kr + k];
    acc = fmaf(xv, wv, acc);
  }
  out[i] = acc;
}

template <int DT, bool WT>
static int lora_down_t(const void* X, int64_t M, int64_t Kr, const void* W2, int R, float pre_s, int do_pre,
                       void* out, float* partial, int64_t partial_elems, unsigned* counters, int ncounters,
                       cudaStream_t st) {
  using T = typename DType<DT>::T;
  if (M <= 16 && R <= kLoraSmallMaxR && Kr <= 0x7fffffff) {
    if (R <= 16) return lora_small_launch<DT, WT, 2>(X, (int)M, (int)Kr, W2, R, pre_s, do_pre, out, st);
    if (R <= 32) return lora_small_launch<DT, WT, 4>(X, (int)M, (int)Kr, W2, R, pre_s, do_pre, out, st);
    return lora_small_launch<DT, WT, 8>(X, (int)M, (int)Kr, W2, R, pre_s, do_pre, out, st);
  }
  if (M <= 16) {
    // split the reduction so that ~128 single-warp CTAs share it
    int64_t ksplit = Kr / 256;
    if (ksplit > 128) ksplit = 128;
    if (ksplit > partial_elems / (M * R)) ksplit = partial_elems / (M * R);
    if (ksplit < 1) ksplit = 1;
    int64_t kchunk = (Kr + ksplit - 1) / ksplit;
    kchunk = (kchunk + 15) / 16 * 16;
    ksplit = (Kr + kchunk - 1) / kchunk;
    if (ksplit > 1 && ncounters < 1) ksplit = 1, kchunk = Kr;
    lora_down_mma_k<DT, WT, 1><<<dim3(1, (unsigned)ksplit), 32, 0, st>>>(
        (const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (int)kchunk, partial, counters, (T*)out);
  } else {
    const int64_t tiles = (M + 15) / 16;
    if (tiles > 0x7fffffff) return RQ_ERR_INVALID;
    const dim3 grid((unsigned)tiles);
    if (R <= 16)
      lora_down_wide_k<DT, WT, 2><<<grid, kWideWarps * 32, 0, st>>>((const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (T*)out);
    else if (R <= 32)
      lora_down_wide_k<DT, WT, 4><<<grid, kWideWarps * 32, 0, st>>>((const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (T*)out);
    else if (R <= 64)
      lora_down_wide_k<DT, WT, 8><<<grid, kWideWarps * 32, 0, st>>>((const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (T*)out);
    else  // r in (64, 128]: 4-warp CTAs over 64 rows, each warp the whole reduction
      lora_down_mma_k<DT, WT, 4><<<dim3((unsigned)((M + 63) / 64), 1), 128, 0, st>>>(
          (const T*)X, M, Kr, (const T*)W2, R, pre_s, do_pre, (int)Kr, partial, counters, (T*)out);
  }
  return check_launch();
}

// Entry used by the layer dispatcher.  `partial`/`counters` may be null (no
// split).  Returns an RQ_* status.
int lora_down(int dt, bool w_transposed, const void* X, int64_t M, int64_t Kr, const void* W2, int R, float pre_s,
              bool do_pre, void* out, float* partial, int64_t partial_elems, unsigned* counters, int ncounters,
              cudaStream_t st) {
  if (R < 1 || R > kLoraMaxR) return RQ_ERR_INVALID;
  if (dt == RQ_F32) {
    const int64_t n = M * R;
    const int64_t grid = (n + 255) / 256;
    if (w_transposed)
      lora_down_f32_k<true><<<(unsigned)grid, 256, 0, st>>>((const float*)X, M, Kr, (const float*)W2, R, pre_s,
                                                            do_pre, (float*)out);
    else
      lora_down_f32_k<false><<<(unsigned)grid, 256, 0, st>>>((const float*)X, M, Kr, (const float*)W2, R, pre_s,
                                                             do_pre, (float*)out);
    return check_launch();
  }
  if (dt == RQ_BF16)
    return w_transposed ? lora_down_t<RQ_BF16, true>(X, M, Kr, W2, R, pre_s, do_pre, out, partial, partial_elems,
                                                     counters, ncounters, st)
                        : lora_down_t<RQ_BF16, false>(X, M, Kr, W2, R, pre_s, do_pre, out, partial, partial_elems,
                                                      counters, ncounters, st);
  if (dt == RQ_F16)
    return w_transposed ? lora_down_t<RQ_F16, true>(X, M, Kr, W2, R, pre_s, do_pre, out, partial, partial_elems,
                                                    counters, ncounters, st)
                        : lora_down_t<RQ_F16, false>(X, M, Kr, W2, R, pre_s, do_pre, out, partial, partial_elems,
                                                     counters, ncounters, st);
  return RQ_ERR_DTYPE;
}

}  // namespace rq
