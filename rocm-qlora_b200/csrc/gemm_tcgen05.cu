// gemm_tcgen05.cu -- prefill/training-shaped fused NF4 dequant GEMM on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory),
// issued as 2-SM MMAs by CTA pairs.
//
// Forward  Y[M, N]  = X[M, K] . deq(W[N, K])^T (+ bias, + LoRA), and the
// transposed variant for backward  dX[M, K] = dY[M, N] . deq(W) (+ LoRA),
// bf16/f16 activations, NF4 weights (plain, fp8 or int8 double-quantized
// scales): the forward for M >= 64 (below that the decode GEMV in slabs of
// 16 rows is faster), dX for every M (token rows past M arrive zero-filled
// by the TMA bounds and are not written).
//
// A cluster of two CTAs (one per SM) computes a 256 (tokens) x BN (outputs)
// tile, BN = 256 or 128, with tcgen05.mma.cta_group::2 (M = 256): each CTA
// holds its 128 token rows of the activation tile and HALF of the weight
// tile (BN/2 outputs), and the pair's two tensor cores share both.  The
// dequantized weight is the expensive operand to produce, so each SM
// dequantizes half of what a one-SM 128 x BN tile would need per FLOP.
// The reduction step is 64 (one quant block a weight row in the forward;
// dX steps over 64 weight rows, whose tile is the MN-major B operand: W's
// own row layout, so its codes come by TMA like the forward's).
// 10 warps a CTA:
//   warp 0   TMA producer of this CTA's activation tile [128 x 64] and
//            weight codes per stage (128-byte swizzle for the activations)
//            and, once, its LoRA tiles: forward
//            t = x.A^T [128 x r] and B [BN/2 x r] (r <= 64, zero-filled to 64
//            by the TMA bounds); dX gt = rnd(dY*s).B [128 x r] and A [r x BN/2]
//            (an MN-major operand of 64-column boxes), into the last ring
//            slot, whose first K-loop fill waits until the LoRA MMAs have
//            read them;
//   warp 1   allocates the pair's tensor memory (base accumulator columns
//            0..BN-1, LoRA accumulator BN..2BN-1, so the epilogue keeps the
//            reference's rounding sequence).  In the leader CTA (rank 0)
//            lane 0 issues every MMA of the pair (kind::f16, K = 16, A
//            K-major from shared memory, B K-major in the forward and
//            MN-major in dX) and commits each stage to the stage-free barriers of
//            BOTH CTAs (tcgen05.commit multicast); in the peer CTA lane 0
//            signals "both of this CTA's tiles of the stage are ready" to the
//            leader with a 16-byte bulk copy into the leader's shared memory
//            whose completion lands on the leader's fullB (no fence in the
//            signalling thread, so the signals pipeline);
//   warps 2-9  dequantize this CTA's half of the weight tile of each stage
//            as the reference's exact bf16/f16(T[code] * scale) values into
//            the swizzled K-major (dX: MN-major) layout, arrive on their
//            CTA's fullB, then
//            run the epilogue on this CTA's 128 rows: tcgen05.ld of both
//            accumulators, bias and LoRA rounding, Y stores.
// Barriers: fullA (own TMA bytes), fullB (own 8 dequant warps; in the
// leader also its producer's expect_tx for the peer's signal), empty (MMA
// commit), lora / lorafwd (the peer's LoRA-tile signal), loradone (commit
// of the LoRA MMAs, both CTAs), acc (final commit, both CTAs).  Grid (2,
// output tiles, token pairs): the clusters that run together share token
// rows, so X stays in L2.  Every wait is
// bounded; a wait that runs out raises the abort flag of both CTAs, each
// CTA drains what it has in flight (bounded), Y is not written, the pair
// meets at a cluster barrier before the tensor memory is released, and the
// kernel-timeout counter records it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "gemv_common.cuh"
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

constexpr int BM = 128;                     // token rows a CTA (a pair: 256)
constexpr int BK = 64;
constexpr int kDqWarps = 8;                 // dequant / epilogue warps
constexpr int kThreads = 64 + kDqWarps * 32;
constexpr uint32_t kABytes = BM * BK * 2;   // 16 KB
constexpr uint32_t kWaitLimit = 1u << 22;   // polls of a bounded drain (each at least kPollNs apart)
constexpr uint32_t kPollNs = 32;
constexpr int kPrefetch = 4;                // dX: stages of block scales a dequant thread holds in registers
constexpr int kLutReps = 16;                // copies of the code-byte table (one per half-warp lane)
constexpr uint32_t kLutBytes = 256 * kLutReps * 8;
constexpr uint32_t kSmemCap = 226 * 1024;   // dynamic shared memory budget (static + margin in the last KB)

// Per-CTA shared-memory plan of a BN-wide pair tile (1 KB aligned offsets);
// I8: int8 weights (64 code bytes a row and stage instead of 32).  The
// LoRA tiles (t / gt and LoRA B / A) are read only by the LoRA MMAs, which
// run before the K loop: they lie in the last ring slot (X and weight
// areas), which the K loop takes over once those MMAs have completed.
template <int BN, bool I8>
struct Tile {
  static constexpr int BNH = BN / 2;                  // weight rows (dX: output columns) a CTA
  static constexpr uint32_t kBBytes = BNH * BK * 2;   // 16 KB / 8 KB
  // this CTA's code bytes of one stage (forward: BNH rows x 32 (64) bytes;
  // dX: 64 rows x BNH / 2 (BNH) bytes)
  static constexpr uint32_t kCBytes = BNH * (I8 ? 64 : 32);
  static constexpr uint32_t kStage = kABytes + kBBytes + kCBytes;
  static constexpr uint32_t kFixed = kLutBytes + 1024 + 1024;  // LUT, sclut, alignment
  static constexpr int kFit = (int)((kSmemCap - kFixed) / kStage);
  static constexpr int kStages = kFit > 6 ? 6 : kFit;
  static constexpr uint32_t kSmA = 0;                               // kStages x 16 KB
  static constexpr uint32_t kSmB = kSmA + kStages * kABytes;        // kStages x kBBytes
  static constexpr uint32_t kSmC = kSmB + kStages * kBBytes;        // kStages x kCBytes (codes by TMA)
  static constexpr uint32_t kSmT = kSmA + (kStages - 1) * kABytes;  // LoRA t (gt) tile: the last slot's X area
  static constexpr uint32_t kSmLB = kSmB + (kStages - 1) * kBBytes; // LoRA B (dX: A) tile: its weight area
  static constexpr uint32_t kSmLut = kSmC + kStages * kCBytes;      // code byte -> (T[lo], T[hi])
  static constexpr uint32_t kSmScl = kSmLut + kLutBytes;            // 256 fp32 second-level values
  static constexpr uint32_t kSmBytes = kSmScl + 1024 + 1024;        // + alignment slack
  static constexpr int kTmemCols = 2 * BN;                          // base + LoRA accumulators
  static_assert(kStages >= 3, "pipeline too shallow");
  static_assert(kSmBytes <= kSmemCap, "shared memory plan too large");
};

struct GemmArgs {
  CUtensorMap xmap;   // X [M][K] (dX: dY [M][N]), box 64 x 128, 128-byte swizzle
  CUtensorMap tmap;   // t [M][r] (dX: gt), box 64 x 128, 128-byte swizzle (r < 64 zero-filled)
  CUtensorMap bmap;   // LoRA B [N][r], box 64 x BN/2 (dX: A [r][K], box 64 x 64), 128-byte swizzle
  CUtensorMap cmap;   // codes uint8 [N][K/2] (int8 [N][K]): forward box 32 (64) x BN/2 (one stage of this
                      // CTA's rows), dX box BN/4 (BN/2) x 64 (one stage's rows, this CTA's columns)
  QWeight w;
  const void* bias;
  int bdt;
  void* y;            // Y [M][N] (dX: dX [M][K])
  int M, N, K, r;
  float s;            // LoRA scaling (dX: 1, gt already carries it)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at shared::cta address `a` in CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(rank));
  return d;
}
__device__ __forceinline__ void st_cluster(uint32_t caddr, int v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(caddr), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Signal a barrier of the peer CTA without a fence in this thread: a 16-byte
// shared-to-peer-shared bulk copy whose completion adds 16 transaction bytes
// to the peer's barrier `cbar` (dst and cbar are shared::cluster addresses).
// The receiving CTA posts the matching expect_tx.  A release-arrive at
// cluster scope would wait for this thread's previous remote operations to
// be acknowledged (about a microsecond a stage).
__device__ __forceinline__ void bulk_signal(uint32_t cdst, uint32_t src, uint32_t cbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], 16, [%2];" ::"r"(cdst),
               "r"(src), "r"(cbar)
               : "memory");
}
// Non-blocking test of a phase (test_wait: the thread is never suspended,
// so it sees the completion as soon as it happens).
template <bool kCluster>
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kCluster)
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  return ok != 0;
}

// The abort state of a CTA pair: this CTA's flag and the peer's (remote).
struct Abort {
  volatile int* mine;
  uint32_t peer;  // shared::cluster address of the peer's flag
  __device__ __forceinline__ bool raised() const { return *mine != 0; }
  __device__ __forceinline__ void raise() const {
    *mine = 1;
    st_cluster(peer, 1);
  }
};

// Potentially blocking test of a phase (try_wait: a thread whose phase is
// not complete is suspended in the barrier until it completes or a
// system-dependent time limit passes, so it neither polls the barrier word
// nor oversleeps the completion).
template <bool kCluster>
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kCluster)
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitNs = 2000000000ull;  // a bounded wait gives up after about 2 s

// Bounded wait for the phase of parity `parity`; false if either CTA of the
// pair gave up (then or earlier).
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (mbar_try<kCluster>(bar, parity)) return true;
  const uint64_t t0 = gtimer_ns();
  while (!ab.raised()) {
    if (mbar_try<kCluster>(bar, parity)) return true;
    if (gtimer_ns() - t0 > kWaitNs) {
      ab.raise();
      atomicAdd(&g_gemm_timeouts, 1u);
      return false;
    }
  }
  return false;
}
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit && !mbar_test<false>(bar, parity); ++i) __nanosleep(kPollNs);
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
// B K-major (or MN-major), M = 256 (the CTA pair), N = BN.
template <int DT, int BN>
__device__ __forceinline__ uint32_t idesc_pair(bool b_mn = false) {
  const uint32_t ab = DT == RQ_BF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(256 >> 4) << 24);
}

__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive on the barrier at shared::cta offset `bar` of each CTA in `mask`
// once every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
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

// Two 32-column loads (base and LoRA accumulators of the same rows) under
// one wait: one tensor-memory round trip instead of two.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, float (&a)[32], float (&b)[32]) {
  uint32_t ra[32], rb[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(ra[0]), "=r"(ra[1]), "=r"(ra[2]), "=r"(ra[3]), "=r"(ra[4]), "=r"(ra[5]), "=r"(ra[6]), "=r"(ra[7]), "=r"(ra[8]), "=r"(ra[9]), "=r"(ra[10]), "=r"(ra[11]), "=r"(ra[12]), "=r"(ra[13]), "=r"(ra[14]), "=r"(ra[15]), "=r"(ra[16]), "=r"(ra[17]), "=r"(ra[18]), "=r"(ra[19]), "=r"(ra[20]), "=r"(ra[21]), "=r"(ra[22]), "=r"(ra[23]), "=r"(ra[24]), "=r"(ra[25]), "=r"(ra[26]), "=r"(ra[27]), "=r"(ra[28]), "=r"(ra[29]), "=r"(ra[30]), "=r"(ra[31]), "=r"(rb[0]), "=r"(rb[1]), "=r"(rb[2]), "=r"(rb[3]), "=r"(rb[4]), "=r"(rb[5]), "=r"(rb[6]), "=r"(rb[7]), "=r"(rb[8]), "=r"(rb[9]), "=r"(rb[10]), "=r"(rb[11]), "=r"(rb[12]), "=r"(rb[13]), "=r"(rb[14]), "=r"(rb[15]), "=r"(rb[16]), "=r"(rb[17]), "=r"(rb[18]), "=r"(rb[19]), "=r"(rb[20]), "=r"(rb[21]), "=r"(rb[22]), "=r"(rb[23]), "=r"(rb[24]), "=r"(rb[25]), "=r"(rb[26]), "=r"(rb[27]), "=r"(rb[28]), "=r"(rb[29]), "=r"(rb[30]), "=r"(rb[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = __uint_as_float(ra[i]);
    b[i] = __uint_as_float(rb[i]);
  }
}

// Read-only global loads pinned where they are written (volatile asm): the
// dequant warps' prefetch of scales must be issued stages ahead of its use,
// not sunk to it by the compiler.
__device__ __forceinline__ uint32_t ldg_pin_u8(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u8 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ldg_pin_f32(const void* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
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

template <int DT, bool DX, int BN, bool I8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) gemm_k(const __grid_constant__ GemmArgs g) {
  using TL = Tile<BN, I8>;
  using T = typename DType<DT>::T;
  constexpr int S = TL::kStages, BNH = TL::BNH;
  constexpr uint32_t kBBytes = TL::kBBytes;
  extern __shared__ __align__(1024) unsigned char dsm[];
  // fullA[S], fullB[S], empty[S], lora, lorafwd, acc, drain, loradone
  __shared__ __align__(8) uint64_t bars[3 * S + 5];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag, a_issued, consumed;
  __shared__ __align__(16) uint32_t sig_src[4], sig_dst[4];  // the 16-byte signal copies (contents unused)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();  // 0: leader (issues the pair's MMAs), 1: peer
  // 1 KB aligned view of the dynamic shared memory (swizzle atoms); the
  // same offsets in both CTAs, which the pair's MMAs rely on
  const uint32_t sraw = smem_u32(dsm);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  unsigned char* sm = dsm + (sbase - sraw);
  const uint32_t fullA0 = smem_u32(bars), fullB0 = fullA0 + 8 * S, empty0 = fullB0 + 8 * S;
  const uint32_t lorabar = empty0 + 8 * S, lorafwd = lorabar + 8, accbar = lorafwd + 8, drainbar = accbar + 8;
  const uint32_t loradone = drainbar + 8;  // the LoRA MMAs have read the last slot (both CTAs)
  const Abort ab{&abort_flag, mapa(smem_u32(&abort_flag), rank ^ 1u)};

  const int M = g.M, N = g.N, K = g.K;
  const int W_out = DX ? K : N;       // output columns
  const int nkb = (DX ? N : K) / BK;  // reduction steps
  const int n0 = blockIdx.y * BN;     // the pair's first output column
  const int nh0 = n0 + (int)rank * BNH;  // this CTA's half: weight rows (forward) / output columns (dX)
  const int m0 = (blockIdx.z * 2 + (int)rank) * BM;  // this CTA's token rows
  const bool has_lora = g.r > 0;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(fullA0 + 8 * i, 1);
      mbar_init(fullB0 + 8 * i, rank == 0 ? kDqWarps + 1 : kDqWarps);  // leader: + its producer's expect_tx
      mbar_init(empty0 + 8 * i, 1);
    }
    mbar_init(lorabar, 1);
    mbar_init(lorafwd, 1);
    mbar_init(accbar, 1);
    mbar_init(drainbar, 1);
    mbar_init(loradone, 1);
    abort_flag = 0;
    a_issued = 0;
    consumed = 0;
    for (int i = 0; i < 4; ++i) sig_src[i] = sig_dst[i] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // whole warp, in both CTAs: the pair's tensor memory
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(TL::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  // code byte v -> (T[v & 15], T[v >> 4]) in kLutReps interleaved copies
  // (entry v, copy c at (v * kLutReps + c) * 8: lane l reads copy l % 16, so
  // the 16 lanes of a half warp hit 16 distinct bank pairs), and the
  // second-level table
  float2* lutp = reinterpret_cast<float2*>(sm + TL::kSmLut);
  float* sclut = reinterpret_cast<float*>(sm + TL::kSmScl);
  for (int i = tid; i < 256 * kLutReps; i += kThreads) {
    const int v = i / kLutReps;
    lutp[i] = make_float2(kNF4[v & 15], kNF4[v >> 4]);
  }
  if (g.w.fmt != RQ_W_NF4)
    for (int v = tid; v < 256; v += kThreads)
      sclut[v] = g.w.fmt == RQ_W_NF4_DQ_FP8 ? e4m3fnuz_to_f32(v) : ieee_div((float)(int8_t)v, 127.0f);
  // both CTAs' barriers initialised and the tensor memory allocated before
  // any cross-CTA arrive, commit or MMA
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;
  const uint32_t fullB_lead = mapa(fullB0, 0);  // the leader's fullB[0] (cluster address)
  const uint32_t sig_lead = mapa(smem_u32(sig_dst), 0);

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      if (has_lora) {
        if (rank == 0) mbar_expect_tx(lorafwd, 16);  // the peer's "LoRA tiles landed" signal
        mbar_expect_tx(lorabar, kABytes + kBBytes);
        tma_2d(sbase + TL::kSmT, &g.tmap, 0, m0, lorabar);
        if (DX) {
#pragma unroll
          for (int j = 0; j < BNH / 64; ++j) tma_2d(sbase + TL::kSmLB + j * 8192, &g.bmap, nh0 + 64 * j, 0, lorabar);
        } else {
          tma_2d(sbase + TL::kSmLB, &g.bmap, 0, nh0, lorabar);
        }
      }
      for (int kb = 0; kb < nkb; ++kb) {
        const int slot = kb % S;
        if (kb >= S && !mbar_wait(empty0 + 8 * slot, ((kb / S) - 1) & 1, ab)) break;
        if (kb == S - 1 && has_lora && !mbar_wait(loradone, 0, ab)) break;  // the LoRA tiles are read
        if (rank == 0) mbar_expect_tx(fullB0 + 8 * slot, 16);  // the peer's "stage ready" signal
        mbar_expect_tx(fullA0 + 8 * slot, kABytes + TL::kCBytes);
        tma_2d(sbase + TL::kSmA + slot * kABytes, &g.xmap, kb * BK, m0, fullA0 + 8 * slot);
        // the stage's codes: forward this CTA's BNH weight rows of block kb;
        // dX weight rows 64 kb.. (the reduction), this CTA's BNH columns
        if (DX)
          tma_2d(sbase + TL::kSmC + slot * TL::kCBytes, &g.cmap, I8 ? nh0 : nh0 / 2, kb * BK, fullA0 + 8 * slot);
        else
          tma_2d(sbase + TL::kSmC + slot * TL::kCBytes, &g.cmap, kb * (I8 ? 64 : 32), nh0, fullA0 + 8 * slot);
        *reinterpret_cast<volatile int*>(&a_issued) = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------- MMA issuer (leader CTA)
      const uint32_t idesc = idesc_pair<DT, BN>(), idesc_mn = idesc_pair<DT, BN>(true);
      bool ok = true;
      if (has_lora) {
        ok = mbar_wait(lorabar, 0, ab) && mbar_wait<true>(lorafwd, 0, ab);
        if (ok) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t db = DX ? sw128_mn_desc(sbase + TL::kSmLB + kk * 2048, 8192)  // rows 16kk.. of A
                                   : sw128_desc(sbase + TL::kSmLB + kk * 32);
            mma_pair(tmem + BN, sw128_desc(sbase + TL::kSmT + kk * 32), db, DX ? idesc_mn : idesc,
                     kk > 0);
          }
          mma_commit_pair(loradone, 3);  // both CTAs' last slot is free once these MMAs have read it
        }
      }
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int slot = kb % S;
        const uint32_t par = (kb / S) & 1;
        if (!mbar_wait(fullA0 + 8 * slot, par, ab) || !mbar_wait<true>(fullB0 + 8 * slot, par, ab)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a = sbase + TL::kSmA + slot * kABytes, b = sbase + TL::kSmB + slot * kBBytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // dX: the weight tile is MN-major (W's own row layout)
          mma_pair(tmem, sw128_desc(a + kk * 32), DX ? sw128_mn_desc(b + kk * 2048, 8192) : sw128_desc(b + kk * 32),
                   DX ? idesc_mn : idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_pair(empty0 + 8 * slot, 3);  // both CTAs' slot is free once these MMAs have read it
        *reinterpret_cast<volatile int*>(&consumed) = kb + 1;
      }
      if (ok && !ab.raised()) mma_commit_pair(accbar, 3);  // every MMA of the tile is complete
    } else if (lane == 0) {
      // ------------------------------ forwarder (peer CTA): tiles landed
      bool ok = true;
      if (has_lora) {
        ok = mbar_wait(lorabar, 0, ab);
        if (ok) bulk_signal(mapa(smem_u32(sig_dst), 0), smem_u32(sig_src), mapa(lorafwd, 0));
      }
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int slot = kb % S;
        const uint32_t par = (kb / S) & 1;
        if (!mbar_wait(fullA0 + 8 * slot, par, ab) || !mbar_wait(fullB0 + 8 * slot, par, ab)) break;
        bulk_signal(sig_lead, smem_u32(sig_src), fullB_lead + 8 * slot);
        *reinterpret_cast<volatile int*>(&consumed) = kb + 1;
      }
    }
  } else {
    // ------------------------------------------------ dequant warps (2..9)
    // Both directions take the stage's codes from its TMA copy and store
    // 16-byte units (8 elements) of 128-byte rows, unit c of row n at
    // (c ^ (n & 7)).  Forward: the K-major tile, TPR threads a tile row
    // (weight row nh0 + frow, the 64 elements of block kb).  dX: the
    // MN-major tile, which is W's own row layout: weight row 64 kb + frow
    // (the reduction index), this CTA's BNH output columns in 64-column
    // chunks of 8 KB; 4 threads a row, BNH / 4 columns each (half or a
    // quarter of one quant block).  For BNH = 128 a quarter warp (the lanes
    // one 16-byte store phase serves) takes 4 rows x 2 column quarters of
    // one chunk, so its 8 stores hit 8 distinct bank groups.
    constexpr int CB = I8 ? 64 : 32;                                    // forward: code bytes of a row and stage
    constexpr int TPR = DX ? 4 : 256 / BNH;                             // threads a row
    constexpr int CW = DX ? (I8 ? BNH / 16 : BNH / 32) : (CB / 4) / TPR;  // code words a thread
    constexpr int RB = DX ? (I8 ? BNH : BNH / 2) : CB;                  // code bytes of a row in the stage
    constexpr int UPT = I8 ? CW / 2 : CW;                               // 16-byte units a thread stores
    const int dt = tid - 64;
    const int fmt = g.w.fmt;
    // first-level scales per block (NF4 / int8) or per row (int8 per-row);
    // otherwise double-quantized (c2 code x c2_scales)
    const bool plain = fmt == RQ_W_NF4 || fmt == RQ_W_INT8, rowsc = fmt == RQ_W_INT8_ROW;
    const int nbk = K / 64;
    int frow, fpart;
    if constexpr (DX && BNH == 128) {
      const int q = lane >> 3, idx = lane & 7;
      frow = 8 * (warp - 2) + 4 * (q >> 1) + (idx & 3);
      fpart = (idx >> 2) + 2 * (q & 1);
    } else {
      frow = dt / TPR;
      fpart = dt % TPR;
    }
    const int dcol = DX ? fpart * (BNH / 4) : 0;  // dX: first of the thread's output columns in the CTA's half
    const uint32_t row_off = (uint32_t)(dcol / 64) * 8192u + (uint32_t)frow * 128u;
    const int ub = DX ? (dcol % 64) / 8 : fpart * UPT;  // the thread's first unit in its row
    const uint32_t lut_lane = smem_u32(lutp) + (uint32_t)(lane & (kLutReps - 1)) * 8;
    // (T[lo], T[hi]) of byte J of `w`: one byte permute, one multiply-add, one 8-byte load
    auto lut_at = [&](uint32_t w, int j) -> float2 {
      const uint32_t addr = __byte_perm(w, 0u, 0x4440u | (uint32_t)j) * (kLutReps * 8) + lut_lane;
      float2 v;
      asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
      return v;
    };
    // sv: the block scale of the thread's elements in stage kb
    auto convert = [&](int kb, float sv) -> bool {
      const int slot = kb % S;
      // lane 0 polls the barrier (the other lanes wait in the shuffle, so
      // the shared-memory pipe the TMA writes through is not flooded with
      // polls), and the warp takes one decision: the stage's TMA (X or dY
      // and this CTA's codes) has landed, which also means the slot's
      // previous MMAs are done (the producer issued it only after they were)
      bool free_slot = true;
      if (lane == 0) free_slot = mbar_wait(fullA0 + 8 * slot, (kb / S) & 1, ab);
      if (!__shfl_sync(0xffffffffu, (int)free_slot, 0)) return false;
      unsigned char* rowp = sm + TL::kSmB + slot * kBBytes + row_off;
      uint32_t cw[CW];  // this thread's code words of the stage (TMA-landed)
      {
        const unsigned char* cs = sm + TL::kSmC + slot * TL::kCBytes + frow * RB + fpart * (CW * 4);
        if constexpr (CW == 8) {
          const uint4 v = *reinterpret_cast<const uint4*>(cs), v2 = *reinterpret_cast<const uint4*>(cs + 16);
          cw[0] = v.x;
          cw[1] = v.y;
          cw[2] = v.z;
          cw[3] = v.w;
          cw[4] = v2.x;
          cw[5] = v2.y;
          cw[6] = v2.z;
          cw[7] = v2.w;
        } else if constexpr (CW == 4) {
          const uint4 v = *reinterpret_cast<const uint4*>(cs);
          cw[0] = v.x;
          cw[1] = v.y;
          cw[2] = v.z;
          cw[3] = v.w;
        } else {
          const uint2 v = *reinterpret_cast<const uint2*>(cs);
          cw[0] = v.x;
          cw[1] = v.y;
        }
      }
      if constexpr (I8) {
        // int8: bf16/f16(float(q) * scale), two words a unit
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
          uint32_t qv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t w = cw[2 * i + (j >> 1)];
            const int b = (j & 1) * 16;
            qv[j] = pack_rn<DT>((float)(int8_t)(w >> b) * sv, (float)(int8_t)(w >> (b + 8)) * sv);
          }
          *reinterpret_cast<uint4*>(rowp + (((ub + i) ^ (frow & 7)) << 4)) = make_uint4(qv[0], qv[1], qv[2], qv[3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
          uint32_t qv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 l = lut_at(cw[i], j);
            qv[j] = pack_rn<DT>(l.x * sv, l.y * sv);
          }
          *reinterpret_cast<uint4*>(rowp + (((ub + i) ^ (frow & 7)) << 4)) = make_uint4(qv[0], qv[1], qv[2], qv[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive(fullB0 + 8 * slot);
      return true;
    };
    if constexpr (DX) {
      // dX: the thread's block scale changes with the weight row, 64 rows a
      // stage; a register ring holds kPrefetch stages of raw scales (static
      // indices: fully unrolled)
      const int blk = (nh0 + dcol) / 64;
      struct DSc {
        uint32_t v;  // plain scale (fp32 bits) or c2 byte
        float s2;    // c2_scale
      };
      auto dfetch = [&](int kb, DSc& q) {
        q.v = 0u;
        q.s2 = 0.0f;
        if (kb >= nkb || blk >= nbk) return;
        const int64_t n = (int64_t)kb * 64 + frow, bi = n * nbk + blk;
        if (plain || rowsc) {
          q.v = __float_as_uint(load_scalar(g.w.scales, g.w.sdt, rowsc ? n : bi));
        } else {
          q.v = ldg_pin_u8(g.w.c2 + bi);
          q.s2 = ldg_pin_f32(g.w.c2s + bi / kDQBlock2);
        }
      };
      DSc ring[kPrefetch];
#pragma unroll
      for (int i = 0; i < kPrefetch; ++i) dfetch(i, ring[i]);
      bool go = true;
      for (int kb = 0; kb < nkb && go; kb += kPrefetch) {
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i) {
          if (go && kb + i < nkb) {
            const float sv = (plain || rowsc) ? __uint_as_float(ring[i].v) : sclut[ring[i].v & 255u] * ring[i].s2;
            go = convert(kb + i, sv);
            dfetch(kb + i + kPrefetch, ring[i]);
          }
        }
      }
    } else {
      // Forward: the codes come with the stage (TMA); the row's block scales
      // are loaded 16 stages at a time, one group ahead of use (raw values in
      // their own registers, so the loads stay in flight until the group is
      // decoded).
      struct Group {
        uint32_t v[16];  // plain scales (fp32 bits) or c2 bytes
        float s2[2];     // c2_scales of the group's first and last block
      };
      const int n = nh0 + frow;
      auto group_fetch = [&](int gi, Group& q) {
        const int s0 = gi * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) q.v[j] = 0u;
        q.s2[0] = q.s2[1] = 0.0f;
        if (s0 >= nkb || n >= N) return;
        const int cnt = nkb - s0 < 16 ? nkb - s0 : 16;
        const int64_t b0 = (int64_t)n * nbk + s0;
        if (plain || rowsc) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < cnt) q.v[j] = __float_as_uint(load_scalar(g.w.scales, g.w.sdt, rowsc ? (int64_t)n : b0 + j));
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < cnt) q.v[j] = ldg_pin_u8(g.w.c2 + b0 + j);
          q.s2[0] = ldg_pin_f32(g.w.c2s + b0 / kDQBlock2);
          q.s2[1] = ldg_pin_f32(g.w.c2s + (b0 + cnt - 1) / kDQBlock2);
        }
      };
      Group gr;  // the next group's raw scales, in flight while 16 stages run
      group_fetch(0, gr);
      bool go = true;
      for (int g0 = 0; g0 < nkb && go; g0 += 16) {
        float sg[16];
        const int64_t b0 = (int64_t)n * nbk + g0;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          sg[j] = (plain || rowsc) ? __uint_as_float(gr.v[j])
                                  : sclut[gr.v[j] & 255u] *
                                        (((b0 + j) / kDQBlock2) != (b0 / kDQBlock2) ? gr.s2[1] : gr.s2[0]);
        group_fetch(g0 / 16 + 1, gr);
#pragma unroll 1
        for (int j = 0; j < 16 && go && g0 + j < nkb; ++j) go = convert(g0 + j, sg[j]);
      }
    }

    // ---------------------------------------------------------- epilogue
    bool ok = true;
    if (lane == 0) ok = mbar_wait(accbar, 0, ab) && !ab.raised();
    ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int quad = warp & 3;  // tensor-memory lanes 32*quad ... are this warp's rows
      const int row = quad * 32 + lane, m = m0 + row;
      const int c_lo = ((warp - 2) >> 2) * (BN / 2);  // warps w and w+4 split the columns
      const bool has_bias = !DX && g.bias != nullptr;
      T* y = static_cast<T*>(g.y);
      for (int cb = c_lo; cb < c_lo + BN / 2; cb += 32) {
        float acc[32], u[32];
        if (has_lora)
          tmem_ld32x2(tmem + ((uint32_t)(quad * 32) << 16) + cb, tmem + ((uint32_t)(quad * 32) << 16) + BN + cb, acc, u);
        else
          tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + cb, acc);
        if (m >= M) continue;
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
            reinterpret_cast<uint4*>(yrow)[q4] =
                make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        } else {
          for (int j = 0; j < 32 && n0 + cb + j < W_out; ++j) {
            const uint32_t w2 = pk[j / 2];
            const uint16_t hbits = (j & 1) ? (uint16_t)(w2 >> 16) : (uint16_t)(w2 & 0xFFFF);
            reinterpret_cast<uint16_t*>(yrow)[j] = hbits;
          }
        }
      }
    }
  }

  // ---------------------------------------------------------- teardown
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1 && lane == 0 && ab.raised()) {
    // Work may still be in flight: the leader waits (bounded) for all of its
    // MMAs; each CTA for the TMA copies its producer issued that nothing
    // waited for, before the shared and tensor memory are released
    if (rank == 0) {
      mma_commit_pair(drainbar, 1);
      mbar_drain(drainbar, 0);
    }
    const int done = *reinterpret_cast<volatile int*>(&consumed), issued = *reinterpret_cast<volatile int*>(&a_issued);
    for (int kb = done; kb < issued; ++kb) mbar_drain(fullA0 + 8 * (kb % S), (kb / S) & 1);
    if (has_lora) mbar_drain(lorabar, 0);
  }
  // the peer's shared memory stays alive until the leader's MMAs are done,
  // and no remote arrive, signal or commit can reach a CTA that has left.
  // On the normal path the leader consumed every signal the peer sent; after
  // an abort the peer's last signals may still be in flight: the leader
  // gives them a bounded time to land between two cluster barriers (both
  // CTAs pass both barriers on every path).
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();
  if (tid == 0 && rank == 0 && ab.raised()) {
    uint64_t t0, t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
      __nanosleep(1000);
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    } while (t1 - t0 < 50000);  // 50 us
  }
  cluster_sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TL::kTmemCols) : "memory");
}


// ------------------------------------------------------------------------
// LoRA down product of the prefill / training paths on the tensor cores:
//   forward  t  = rnd(X[M, Kr] . A^T)          A  [R, Kr] (K-major operand)
//   dX       gt = rnd(s . (dY[M, Kr] . B))      B  [Kr, R] (MN-major operand)
// (dX only for s a power of two: then rnd(dY*s) = dY*s exactly and scaling
// the fp32 sum is exact, so this equals the reference's rnd(rnd(dY*s).B)).
// A cluster of SK CTAs shares a 128-row tile, CTA k reducing the k-th slice
// of the 64-wide steps; each accumulates in tensor memory (M=128, N=RP),
// parks its fp32 partial in shared memory, and the cluster's rank 0 sums
// the partials in rank order through distributed shared memory (fixed
// order: deterministic), rounds and stores.  6 warps: TMA producer, MMA
// issuer (+ tensor memory), 4 epilogue warps (one TMEM lane quarter each).
constexpr int kLdStages = 3;
constexpr int kLdThreads = 192;
constexpr uint32_t kLdX = 128 * 64 * 2;   // X tile, 16 KB
constexpr uint32_t kLdW = 64 * 64 * 2;    // A / B tile, 8 KB (rows past R zero-filled)
constexpr int kLdRedStride = 64 + 4;      // floats a row of the parked partial (bank spread)
constexpr uint32_t kLdSmem = kLdStages * (kLdX + kLdW) + 128 * kLdRedStride * 4 + 1024;

struct LoraDownArgs {
  CUtensorMap xmap;   // X / dY [M][Kr], box 64 x 128, 128-byte swizzle
  CUtensorMap wmap;   // A [R][Kr] box 64 x RP (forward), B [Kr][R] box 64 x 64 (dX), 128-byte swizzle
  void* out;          // [M][R] activation dtype
  int M, Kr, R, rp, sk;
  float s;            // dX scale (a power of two), 1 forward
};

template <int DT, bool WT>
__global__ void __launch_bounds__(kLdThreads, 1) lora_down_tc_k(const __grid_constant__ LoraDownArgs g) {
  using T = typename DType<DT>::T;
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t bars[2 * kLdStages + 1];  // full[S], empty[S], acc
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag, issued, consumed;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t sraw = smem_u32(dsm), sbase = (sraw + 1023u) & ~1023u;
  unsigned char* sm = dsm + (sbase - sraw);
  float* red = reinterpret_cast<float*>(sm + kLdStages * (kLdX + kLdW));
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kLdStages, accbar = empty0 + 8 * kLdStages;
  // waits give up on this CTA's flag only (the cluster meets at barriers the
  // whole cluster always reaches)
  const Abort ab{&abort_flag, mapa(smem_u32(&abort_flag), rank)};
  const int m0 = (int)(blockIdx.x / g.sk) * 128;
  const int nsteps = g.Kr / 64;
  const int s0 = nsteps * (int)rank / g.sk, s1 = nsteps * ((int)rank + 1) / g.sk;
  const uint32_t tcols = g.rp <= 32 ? 32u : 64u;

  if (tid == 0) {
    for (int i = 0; i < kLdStages; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    mbar_init(accbar, 1);
    abort_flag = 0;
    issued = 0;
    consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      for (int st = s0; st < s1; ++st) {
        const int i = st - s0, slot = i % kLdStages;
        if (i >= kLdStages && !mbar_wait(empty0 + 8 * slot, ((i / kLdStages) - 1) & 1, ab)) break;
        const uint32_t xs = sbase + slot * (kLdX + kLdW), ws = xs + kLdX;
        mbar_expect_tx(full0 + 8 * slot, kLdX + (WT ? kLdW : (uint32_t)g.rp * 128));
        tma_2d(xs, &g.xmap, st * 64, m0, full0 + 8 * slot);
        if (WT)
          tma_2d(ws, &g.wmap, 0, st * 64, full0 + 8 * slot);
        else
          tma_2d(ws, &g.wmap, st * 64, 0, full0 + 8 * slot);
        *reinterpret_cast<volatile int*>(&issued) = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t ab16 = DT == RQ_BF16 ? 1u : 0u;
      const uint32_t idesc = (1u << 4) | (ab16 << 7) | (ab16 << 10) | ((WT ? 1u : 0u) << 16) |
                             ((uint32_t)(g.rp >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      for (int st = s0; st < s1; ++st) {
        const int i = st - s0, slot = i % kLdStages;
        if (!mbar_wait(full0 + 8 * slot, (i / kLdStages) & 1, ab)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t xs = sbase + slot * (kLdX + kLdW), ws = xs + kLdX;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t db = WT ? sw128_mn_desc(ws + kk * 2048, 8192) : sw128_desc(ws + kk * 32);
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
              "l"(sw128_desc(xs + kk * 32)), "l"(db), "r"(idesc), "r"((i > 0 || kk > 0) ? 1u : 0u)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(empty0 +
                                                                                                      8 * slot)
                     : "memory");
        *reinterpret_cast<volatile int*>(&consumed) = i + 1;
      }
      // all of this CTA's MMAs (none when its slice is empty) are complete
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(accbar)
                   : "memory");
    }
  } else {
    // ---------------------------------------------- epilogue warps (2..5)
    const int quad = warp & 3, row = quad * 32 + lane;
    bool ok = true;
    if (lane == 0) ok = mbar_wait(accbar, 0, ab) && !ab.raised();
    ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    float* myrow = red + row * kLdRedStride;
    for (int c = 0; c < g.rp; c += 32) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c + j < 64) myrow[c + j] = (ok && s1 > s0) ? v[j] : 0.0f;
    }
  }
  // the partials are parked: rank 0 sums them in rank order
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  cluster_sync();
  if (rank == 0 && warp >= 2) {
    const int quad = warp & 3, row = quad * 32 + lane, m = m0 + row;
    const uint32_t mine = smem_u32(red + row * kLdRedStride);
    T* out = static_cast<T*>(g.out);
    for (int c = 0; c < g.R; c += 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < g.sk; ++q) {
        float4 v;
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "r"(mapa(mine + c * 4, (uint32_t)q)));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      if (m < g.M) {
        const float o[4] = {acc.x * g.s, acc.y * g.s, acc.z * g.s, acc.w * g.s};
        for (int j = 0; j < 4 && c + j < g.R; ++j) out[(size_t)m * g.R + c + j] = DType<DT>::from_f32(o[j]);
      }
    }
  }
  // peers stay alive until rank 0 has read their partials; drain after an abort
  __syncwarp();
  cluster_sync();
  if (warp == 1 && lane == 0 && ab.raised()) {
    mbar_drain(accbar, 0);
    const int done = *reinterpret_cast<volatile int*>(&consumed), n = *reinterpret_cast<volatile int*>(&issued);
    for (int i = done; i < n; ++i) mbar_drain(full0 + 8 * (i % kLdStages), (i / kLdStages) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

}  // namespace

// ---------------------------------------------------------------- host side

bool gemm_supported(const LinearArgs& a, bool dx) {
  if (a.M < (dx ? 1 : 64) || a.w.K % 64) return false;
  if (is_nf4_fmt(a.w.fmt) || a.w.fmt == RQ_W_INT8) {
    if (a.w.bs != 64) return false;  // one quant block a row and step
  } else if (a.w.fmt != RQ_W_INT8_ROW) {
    return false;
  }
  if (dx && a.w.N % 64) return false;  // dX reduces over N in steps of 64 rows
  if (a.xdt != RQ_BF16 && a.xdt != RQ_F16) return false;
  if (a.r > 64 || (a.r > 0 && a.r % 8)) return false;
  if ((uintptr_t)a.x % 16 || (uintptr_t)a.w.q % 16) return false;
  if (a.r > 0 && (uintptr_t)a.lora_b % 16) return false;
  if ((dx ? a.w.K : a.w.N) > 65535LL * 128 || a.M > 65535LL * 256) return false;  // grid y and z
  return a.w.N <= 0x7fffffff && a.w.K <= 0x7fffffff && a.M <= 0x7fffffff;
}

template <int DT, bool DX, int BN, bool I8>
static int gemm_run(const GemmArgs& g, uint64_t wout, uint64_t M, cudaStream_t st) {
  constexpr uint32_t smem = Tile<BN, I8>::kSmBytes;
  const void* kern = (const void*)gemm_k<DT, DX, BN, I8>;
  const int rc = ensure_smem_limit(kern, smem);
  if (rc != RQ_OK) return rc;
  // CTA pairs along x, output tiles along y, 256-row token pairs along z
  // (consecutive clusters share X rows); the cluster shape is given at
  // launch as well
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2u, (unsigned)((wout + BN - 1) / BN), (unsigned)((M + 255) / 256));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_k<DT, DX, BN, I8>, g);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return check_launch();
}

template <bool I8>
static int gemm_pick(int xdt, bool dx, int bn, const GemmArgs& g, uint64_t wout, uint64_t M, cudaStream_t st) {
  if (xdt == RQ_BF16) {
    if (dx)
      return bn == 256 ? gemm_run<RQ_BF16, true, 256, I8>(g, wout, M, st) : gemm_run<RQ_BF16, true, 128, I8>(g, wout, M, st);
    return bn == 256 ? gemm_run<RQ_BF16, false, 256, I8>(g, wout, M, st)
                     : gemm_run<RQ_BF16, false, 128, I8>(g, wout, M, st);
  }
  if (dx) return bn == 256 ? gemm_run<RQ_F16, true, 256, I8>(g, wout, M, st) : gemm_run<RQ_F16, true, 128, I8>(g, wout, M, st);
  return bn == 256 ? gemm_run<RQ_F16, false, 256, I8>(g, wout, M, st) : gemm_run<RQ_F16, false, 128, I8>(g, wout, M, st);
}

// Tile width: 256 outputs a pair unless that leaves SMs idle, then 128.
static int pick_bn(uint64_t wout, uint64_t M) {
  const uint64_t ctas256 = 2 * ((wout + 255) / 256) * ((M + 255) / 256);
  return ctas256 < (uint64_t)num_sms() ? 128 : 256;
}

// Shared launch of both variants: `a_op` is X (forward) or dY (dX), `t` the
// down product (t or gt), `bmat` LoRA B (forward) or A (dX).
static int gemm_launch(const LinearArgs& a, bool dx, const void* a_op, const void* t, cudaStream_t st) {
  GemmArgs g;
  const uint64_t M = (uint64_t)a.M, N = (uint64_t)a.w.N, K = (uint64_t)a.w.K, r = (uint64_t)(a.r > 0 ? a.r : 8);
  const uint64_t red = dx ? N : K, wout = dx ? K : N;
  const int bn = pick_bn(wout, M);
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
    } else {  // B [N][r]: a CTA's bn/2 rows
      const uint64_t db[3] = {r, N, 1}, sb[2] = {r * 2, 0};
      const uint32_t bb[3] = {BK, (uint32_t)(bn / 2), 1};
      rc = tensor_map_encode(ty, swz, 2, a.lora_b, db, sb, bb, &g.bmap);
    }
    if (rc != RQ_OK) return rc;
  } else {
    g.tmap = g.xmap;
    g.bmap = g.xmap;
  }
  const bool i8 = !is_nf4_fmt(a.w.fmt);
  {  // codes [N][K/2] (int8: [N][K]) bytes; a stage's box: forward a CTA's
     // bn/2 rows x 32 (64) bytes, dX 64 rows x the bytes of a CTA's bn/2 columns
    const uint64_t rowb = i8 ? K : K / 2;
    const uint64_t d[3] = {rowb, N, 1}, sd[2] = {rowb, 0};
    const uint32_t half = (uint32_t)(bn / 2);
    const uint32_t b[3] = {dx ? (i8 ? half : half / 2) : (i8 ? 64u : 32u), dx ? 64u : half, 1};
    const int rc = tensor_map_encode(CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_NONE, 2, a.w.q, d, sd, b,
                                     &g.cmap);
    if (rc != RQ_OK) return rc;
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
  return i8 ? gemm_pick<true>(a.xdt, dx, bn, g, wout, M, st) : gemm_pick<false>(a.xdt, dx, bn, g, wout, M, st);
}

int gemm_forward(const LinearArgs& a, const void* tdown, cudaStream_t st) { return gemm_launch(a, false, a.x, tdown, st); }

// The tensor-core down product for M >= 256 (see lora_down_tc_k); returns
// RQ_ERR_UNSUPPORTED (nothing launched) for arguments it does not take, and
// the caller runs lora_down instead.
int lora_down_tc(int dt, bool wt, const void* X, int64_t M, int64_t Kr, const void* W2, int R, float pre_s,
                 bool do_pre, void* out, cudaStream_t st) {
  if ((dt != RQ_BF16 && dt != RQ_F16) || M < 256 || M > 0x7fffffff || R < 8 || R > 64 || R % 8 || Kr % 64 ||
      Kr > 0x7fffffff)
    return RQ_ERR_UNSUPPORTED;
  float s = 1.0f;
  if (do_pre) {  // exact only for a power-of-two scale
    int e = 0;
    if (!(pre_s > 0.0f) || frexpf(pre_s, &e) != 0.5f) return RQ_ERR_UNSUPPORTED;
    s = pre_s;
  }
  if ((uintptr_t)X % 16 || (uintptr_t)W2 % 16 || (uintptr_t)out % 4) return RQ_ERR_UNSUPPORTED;
  LoraDownArgs g;
  const int ty = CU_TENSOR_MAP_DATA_TYPE_UINT16, swz = CU_TENSOR_MAP_SWIZZLE_128B;
  const int rp = (R + 15) / 16 * 16;
  {
    const uint64_t d[3] = {(uint64_t)Kr, (uint64_t)M, 1}, sd[2] = {(uint64_t)Kr * 2, 0};
    const uint32_t b[3] = {64, 128, 1};
    const int rc = tensor_map_encode(ty, swz, 2, X, d, sd, b, &g.xmap);
    if (rc != RQ_OK) return rc;
  }
  {
    int rc;
    if (wt) {  // B [Kr][R]: 64 K rows x 64 columns (past R zero-filled), MN-major operand
      const uint64_t d[3] = {(uint64_t)R, (uint64_t)Kr, 1}, sd[2] = {(uint64_t)R * 2, 0};
      const uint32_t b[3] = {64, 64, 1};
      rc = tensor_map_encode(ty, swz, 2, W2, d, sd, b, &g.wmap);
    } else {  // A [R][Kr]: rp rows (past R zero-filled) x 64 K
      const uint64_t d[3] = {(uint64_t)Kr, (uint64_t)R, 1}, sd[2] = {(uint64_t)Kr * 2, 0};
      const uint32_t b[3] = {64, (uint32_t)rp, 1};
      rc = tensor_map_encode(ty, swz, 2, W2, d, sd, b, &g.wmap);
    }
    if (rc != RQ_OK) return rc;
  }
  const int64_t tiles = (M + 127) / 128, nsteps = Kr / 64;
  // split-K depth: the deepest that keeps the grid in one round (two CTAs
  // fit an SM); one more (the rounded-up share) left a second round of a
  // few clusters that doubled the call (M = 8192: 320 CTAs for 296 slots)
  int64_t sk = 2 * (int64_t)num_sms() / tiles;
  if (sk > 8) sk = 8;
  if (sk > nsteps) sk = nsteps;
  if (sk < 1) sk = 1;
  g.out = out;
  g.M = (int)M;
  g.Kr = (int)Kr;
  g.R = R;
  g.rp = rp;
  g.sk = (int)sk;
  g.s = s;
  const void* kern = dt == RQ_BF16 ? (wt ? (const void*)lora_down_tc_k<RQ_BF16, true> : (const void*)lora_down_tc_k<RQ_BF16, false>)
                                   : (wt ? (const void*)lora_down_tc_k<RQ_F16, true> : (const void*)lora_down_tc_k<RQ_F16, false>);
  int rc = ensure_smem_limit(kern, kLdSmem);
  if (rc != RQ_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * sk), 1, 1);
  cfg.blockDim = dim3(kLdThreads, 1, 1);
  cfg.dynamicSmemBytes = kLdSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)sk;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void* args[] = {&g};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return check_launch();
}

// dX: a.x is dY [M][N], gt = rnd(rnd(dY*s).B) [M][r], a.y the dX output.
int gemm_dx(const LinearArgs& a, const void* gt, cudaStream_t st) {
  if (a.r > 0 && ((uintptr_t)a.lora_a % 16 || (a.w.K * 2) % 16)) return RQ_ERR_ALIGN;
  return gemm_launch(a, true, a.x, gt, st);
}

}  // namespace rq
