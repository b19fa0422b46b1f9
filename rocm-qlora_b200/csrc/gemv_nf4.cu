// gemv_nf4.cu -- decode-shaped (M <= 16) fused dequant + GEMV + LoRA on a
// TMA ring.
//
// Y[M, N] = X[M, K] . deq(W[N, K])^T with the LoRA / bias epilogue of
// LoRALinear.forward, for NF4 weights with per-block scales or with
// double-quantized (fp8 e4m3fnuz or int8) scales, and for int8 weights with
// per-block or per-row scales (template WK: a stage row is 512 code bytes,
// each int8 pair becomes its exact bf16 / f16 pair by two conversions and
// one packed convert, no table; per-row scales multiply the row sum in the
// epilogue, as the register-fed int8 kernel of gemv_kernels.cu does).
//
// The code stream (N*K/2 bytes) is the cost; the shared-memory data path
// (128 bytes per clock per SM) is the second limit.  So:
//
//  * CTA i owns 16-row tiles [i*TPC, (i+1)*TPC) of W (one contiguous byte
//    range), processed in `chunks` passes of NT tiles; every CTA but the last
//    holds the same count, so one tensor-map box size serves all;
//  * one producer thread streams the pass through a shared-memory ring of S
//    stages with TMA: stage s holds 64-blocks [8s, 8s+8) of the pass's rows
//    and X's matching 512 columns (one box, M rows); stage completion and
//    release go through mbarriers (transaction bytes / consumer-warp
//    arrivals).  The codes come as one 3-D box [128 bytes][2][rows] when
//    K % 256 == 0 (each row's 256 contiguous bytes in one request pair, the
//    DRAM-friendly shape), else as two 2-D 128-byte-wide boxes; both with
//    128-byte swizzle;
//  * 16 consumer warps: warps w and w + 8 multiply block 8s + w of the
//    stage, w for the pass's even tiles and w + 8 for the odd ones (two warps
//    per block column: twice the warps in flight to cover the latency of the
//    table lookups and MMA chains, half the accumulators each); the block
//    columns meet in shared memory at the end in a fixed order
//    (deterministic);
//  * the multiply is mma.sync m16n8k16 with the weights as the A operand (16
//    rows x 16 k) and X as B (8 tokens; two groups for M > 8), so M <= 8
//    costs one MMA per 256 weights.  With the swizzle, the 8-byte code reads
//    of a half warp hit 16 distinct 8-byte bank pairs: in the 3-D layout
//    (shared row 2*r + half) directly, in the 2-D layout (shared row r) when
//    MMA row g reads tile row 2*(g & 3) + (g >> 2) (and +8);
//  * a code byte becomes its 16-bit operand pair through a 256-entry table
//    replicated 32 times (entry v, copy l at v*128 + l*4: lane l reads bank
//    l), one byte permute, one multiply-add and one shared load;
//  * block scales: the producer bulk-copies each pass's raw scale bytes
//    (c2 codes, or the plain per-block scales) into shared memory first; the
//    consumers decode them (fp8/int8 second level times c2_scales) into
//    fragment order; the scale multiplies each block's fp32 partial.
//
// Launch chain: this kernel is always launched as the programmatic dependent
// of the kernel before it in the stream, and triggers its own dependent at
// its start.  A CTA therefore starts as soon as an SM is free -- typically
// the moment the previous layer's CTA there exits -- and streams what no
// kernel of the chain writes (codes, scales, c2 / c2_scales, LoRA B) into
// its ring straight away.  Everything another kernel may still be writing
// is read after griddepcontrol.wait, which returns once the grid before
// this one has finished and its writes are visible: X (without an adapter
// the producer waits after the first ring fill of codes, then issues X for
// those stages), x.A^T and the bias (the epilogue), and with the fused
// gather the flags and counters of the calls before (without an adapter
// the whole kernel waits first).  With LoRA the grid before is the layer's down-product
// kernel; it lets this one launch only after its own griddepcontrol.wait,
// so X is complete at launch and is streamed with the codes from the first
// stage, while the down product runs beside the main loop.
//
// All waits are bounded: a wait that runs out raises the CTA's abort flag,
// the CTA lets its issued copies land (bounded) and returns without writing
// Y, and the event counts in a device counter read by
// rq_take_kernel_timeouts().
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "gemv_common.cuh"

namespace rq {

constexpr int kStageBlocks = 8;                   // 64-blocks per stage (one per consumer warp pair)
constexpr int kNfSplit = 2;                       // consumer warps per block column (they split the stages)
constexpr int kNfWarps = kStageBlocks * kNfSplit;  // consumer warps
constexpr int kNfThreads = kNfWarps * 32;
constexpr int kNfBlockThreads = kNfThreads + 32;  // + the producer warp
constexpr uint32_t kWaitLimit = 1u << 22;         // polls of a barrier before a wait gives up
// Code table: 256 entries x 32 copies (one per lane) of the operand pair
// (T[v & 15], T[v >> 4]), rounded to the activation dtype; in the exact
// mode each copy is the pair of fp32 levels (8 bytes).
__host__ __device__ constexpr uint32_t lut_bytes(bool exact) { return 256u * 32u * (exact ? 8u : 4u); }
constexpr size_t kNfSmemMax = 227 * 1024 - 256;   // dynamic shared memory (static: the barriers)
constexpr int kNfMaxNT1 = 6;                      // 16-row tiles per pass, M <= 8
constexpr int kNfMaxNT2 = 5;                      // 16-row tiles per pass, M > 8
constexpr int kNfMaxSlots = 8;                    // ring stages
// The two consumer warps of a block column may split the stages (each holds
// all the pass's tiles: half the per-stage waits and bookkeeping a tile)
// unless a 16-token pass has 4 or more tiles, whose accumulators would not
// fit in registers; they split the tiles then, and when the ring is shorter
// than 4 stages (gemv_nf4_forward decides).
__host__ __device__ constexpr bool nf4_stage_split(int mg, int nt) { return !(mg == 2 && nt >= 4); }

// Bounded waits that ran out (a kernel that stopped early).
__device__ unsigned int g_kernel_timeouts;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The end of a gathering call, run by one warp of every CTA after a CTA
// barrier has ordered the CTA's stores before it.  Lane 0 arrives with an
// acquire-release atomic (GPU scope); the last CTA to arrive has thereby
// acquired every CTA's stores.  Its warp advances the epoch and publishes it
// to every rank at once, lane q to rank q's flag slot for this rank: each
// lane fences at system scope (cumulative, after the warp barrier that
// follows lane 0's acquire: every CTA's stores to all ranks' Y become
// visible before the flag) and stores the flag relaxed.  Lane q then waits,
// at most about 2 s, until rank q's flag here holds the epoch (acquire at
// system scope): from then on every rank's shard of this call is in this
// rank's Y.  The arrival counter goes back to zero for the next call.
__device__ void gather_arrive(const RqGather& g, int lane) {
  uint32_t* ctrl = g.ctrl;
  uint32_t arrived = 0;
  if (lane == 0)
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(arrived) : "l"(ctrl) : "memory");
  arrived = __shfl_sync(0xffffffffu, arrived, 0);
  if (arrived != gridDim.x - 1) return;
  const uint32_t epoch = *reinterpret_cast<volatile const uint32_t*>(ctrl + 1) + 1;
  __syncwarp();
  if (lane == 0) {
    ctrl[0] = 0;
    ctrl[1] = epoch;
  }
  for (int q = lane; q < g.world; q += 32) {
    uint32_t* f = g.flags[q] + g.rank;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
  const uint64_t t0 = global_ns();
  bool ok = true;
  for (int q = lane; q < g.world; q += 32) {
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(g.my_flags + q) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (global_ns() - t0 > 2000000000ull) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0) {
    ctrl[2] = 1;
    atomicAdd(&g_kernel_timeouts, 1u);
  }
}

// Entry of a gathering call: its epoch (the value the call publishes at
// its end) is the control block's epoch + 1; every CTA reads it at its
// start, before any CTA can have arrived, so all CTAs read the same value.
// CTA 0 announces to every rank that this rank has entered the call (its
// stream has passed every earlier consumer of its Y), lane q to rank q.
// The announcement orders nothing (every earlier kernel of this stream has
// finished), so the stores are relaxed: no fence on the kernel's start.
__device__ uint32_t gather_epoch_of(const RqGather& g) {
  return *reinterpret_cast<volatile const uint32_t*>(g.ctrl + 1) + 1;
}
__device__ void gather_enter(const RqGather& g, uint32_t epoch, int lane) {
  if (blockIdx.x != 0) return;
  for (int q = lane; q < g.world; q += 32) {
    uint32_t* f = g.flags[q] + g.world + g.rank;
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
}

// Before a CTA stores its outputs into the other ranks' Y: wait (at most
// about 2 s, one lane per rank) until every rank has entered this call, so
// that no rank's copy of Y is overwritten while that rank may still be
// reading the previous call's result.  Run by one full warp; returns false
// (and raises the error flag) if a rank did not enter in time.
__device__ bool gather_entered(const RqGather& g, uint32_t epoch, int lane) {
  bool ok = true;
  const uint64_t t0 = global_ns();
  for (int q = lane; q < g.world; q += 32) {
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(g.my_flags + g.world + q) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (global_ns() - t0 > 2000000000ull) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0) {
    g.ctrl[2] = 1;
    atomicAdd(&g_kernel_timeouts, 1u);
  }
  return ok;
}

struct Nf4Args {
  CUtensorMap wmap;  // codes: 3-D uint8 [N][K/256][128], box 128 x 2 x NT*16 (wide),
                     // else 2-D uint8 [N][K/2], box 128 x NT*16; 128-byte swizzle
  CUtensorMap xmap;  // X: 32-bit pairs [M][K/2], box 256 x M
  GemvArgs a;
  int tiles;         // 16-row tiles of W
  int tpc;           // tiles per CTA (NT * chunks)
  int chunks;        // passes per CTA
  int sp;            // floats per block row of the staged scales (NT * 16 + 2)
  int esz;           // bytes per raw scale (1: c2 codes; 2/4: plain scales)
  int wide;          // 1: 3-D code box (K % 256 == 0)
  int stage_split;   // 1: the two warps of a block column split the stages (nf4_stage_split)
  int wk;            // code format: 0 NF4 family, 1 int8 blockwise, 2 int8 per-row
  int xsafe;         // 1: X is complete when this grid launches (it follows the
                     // down-product kernel, which lets it launch only after
                     // its own griddepcontrol.wait), so X is loaded at once
  int slots;         // ring stages S
  int sw;            // stages a scale window (0: the pass's scales decoded at once)
  uint32_t slot_bytes;  // 2 * NT*16*128 (codes) + M*1024 (X), a multiple of 1024
  uint32_t ring_off;    // dynamic offsets: ring (rounded up to 1024 in the shared window),
  uint32_t red_off;     //   partial sums (0: the ring itself),
  uint32_t sc_off;      //   decoded scales of a pass,
  uint32_t raw_off;     //   raw scale bytes of a pass, c2_scales of a pass,
  uint32_t aux_off;     //   256-entry second-level scale table,
  uint32_t tl_off;      //   staged x.A^T
  uint32_t stg_off;     //   a pass's outputs [M][NT*16] (gathering calls)
  uint32_t bsm_off;     //   the pass's rows of LoRA B [NT*16][r]
  int bsm;              // 1: B's rows are bulk-copied with the raw scales (one pass, r % 8 == 0)
};

// NF4 level c (the values of kNF4) from immediates: no memory access, so the
// table build does not wait on a cold constant cache.
__device__ __forceinline__ float nf4_level_imm(int c) {
  float v = -1.0f;
  v = c == 1 ? -0.6961928009986877f : v;
  v = c == 2 ? -0.5250730514526367f : v;
  v = c == 3 ? -0.39491748809814453f : v;
  v = c == 4 ? -0.28444138169288635f : v;
  v = c == 5 ? -0.18477343022823334f : v;
  v = c == 6 ? -0.09105003625154495f : v;
  v = c == 7 ? 0.0f : v;
  v = c == 8 ? 0.07958029955625534f : v;
  v = c == 9 ? 0.16093020141124725f : v;
  v = c == 10 ? 0.24611230194568634f : v;
  v = c == 11 ? 0.33791524171829224f : v;
  v = c == 12 ? 0.44070982933044434f : v;
  v = c == 13 ? 0.5626170039176941f : v;
  v = c == 14 ? 0.7229568362236023f : v;
  v = c == 15 ? 1.0f : v;
  return v;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Operand pair of code byte KB of `word` for this lane (lanesel: shared
// address of the table plus lane*4).
template <int KB>
__device__ __forceinline__ uint32_t lut2(uint32_t word, uint32_t lanesel) {
  return lds_u32(__byte_perm(word, 0u, 0x4440u | KB) * 128u + lanesel);
}
// fp32 level pair (T[lo nibble], T[hi nibble]) of code byte KB of `word` for
// this lane (lanesel: shared address of the table plus lane*8)
template <int KB>
__device__ __forceinline__ uint2 lut4(uint32_t word, uint32_t lanesel) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "r"(__byte_perm(word, 0u, 0x4440u | KB) * 256u + lanesel));
  return v;
}

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
// Waits for the phase of `bar` with the given parity, at most kWaitLimit
// polls; a wait that runs out raises the CTA's abort flag (every later wait
// then returns at once) and counts in g_kernel_timeouts.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_test(bar, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1;
  atomicAdd(&g_kernel_timeouts, 1u);
  return false;
}

// ---- LoRA down product fused into the grid (GemvArgs::fuse_down)
//
// The grid's first kNfDownCtas CTAs compute the partial sums of
// t = x_lora . A^T while the other CTAs run the GEMV.  Every warp of those
// CTAs takes 16-column k-steps round robin (mma.sync m16n8k16: tokens x k
// times k x adapter rows, fp32 accumulators; the loads of two k-steps are in
// flight before their MMAs), and each CTA sums its warps in warp order into
// its fp32 partial [M][r] in the workspace, then adds 1 to counters[0] with
// release semantics.  Every GEMV CTA waits (acquire, bounded) until all
// kNfDownCtas partials are in, sums them in CTA order and rounds once to
// the activation dtype (the reference's lora_A(x) output) -- the same value
// in every CTA.  The last GEMV CTA to finish zeroes counters[0] and [2]
// again, so the counter area is zero at rest.  No CTA of this grid waits on
// a later grid, and this grid's dependent launches only once every CTA of
// it is resident, so the down CTAs always run.
__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Waits (at most kWaitLimit polls) until *p >= v; false if it gave up
// (counted in g_kernel_timeouts).
__device__ __forceinline__ bool count_wait(const unsigned* p, uint32_t v) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (ld_acquire_gpu(p) >= v) return true;
    __nanosleep(32);
  }
  atomicAdd(&g_kernel_timeouts, 1u);
  return false;
}

// shared memory of the down role: [warps][16 tokens][8 * ceil(r / 8)] fp32
__host__ __device__ constexpr size_t down_smem(int r) {
  return (size_t)(kNfBlockThreads / 32) * 16 * (size_t)(8 * ((r + 7) / 8)) * sizeof(float);
}

template <int DT, int NJ>
__device__ __forceinline__ void down_kstep(const typename DType<DT>::T* x0, const typename DType<DT>::T* x1,
                                           const typename DType<DT>::T* A, int K, int r, int nj, bool r0, bool r1,
                                           int k0, int g, int t, uint32_t (&a)[4], uint32_t (&b)[NJ][2]) {
  // x through L2 (the grid before may have written it), A through the
  // read-only path (a weight)
  a[0] = r0 ? __ldcg(reinterpret_cast<const unsigned*>(x0 + k0)) : 0u;
  a[1] = r1 ? __ldcg(reinterpret_cast<const unsigned*>(x1 + k0)) : 0u;
  a[2] = r0 ? __ldcg(reinterpret_cast<const unsigned*>(x0 + k0 + 8)) : 0u;
  a[3] = r1 ? __ldcg(reinterpret_cast<const unsigned*>(x1 + k0 + 8)) : 0u;
#pragma unroll
  for (int jt = 0; jt < NJ; ++jt) {
    const int j = jt * 8 + g;
    const bool ok = jt < nj && j < r;
    const unsigned* ar = reinterpret_cast<const unsigned*>(A + (size_t)(ok ? j : 0) * K + k0 + 2 * t);
    b[jt][0] = ok ? __ldg(ar) : 0u;
    b[jt][1] = ok ? __ldg(ar + 4) : 0u;
  }
}

// NJ: 8-row tiles of A held (nj <= NJ); with NJ <= 4 the loads of two
// k-steps are in flight before their MMAs
template <int DT, int NJ>
__device__ __noinline__ void down_role(const GemvArgs& p, unsigned char* smem) {
  using T = typename DType<DT>::T;
  constexpr int KB = NJ <= 4 ? 2 : 1;
  constexpr int kW = kNfBlockThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int M = (int)p.M, K = (int)p.w.K, r = p.r, nj = (r + 7) >> 3, RP = 8 * nj;
  const T* X = static_cast<const T*>(p.lora_x);
  const T* A = static_cast<const T*>(p.lora_a);
  const int d = blockIdx.x, W = kNfDownCtas * kW, nks = K >> 4;
  // A is a weight: start this CTA's lines of it towards L2 before the wait
  for (int e = tid; e < r * kW; e += kNfBlockThreads) {
    const int j = e / kW, w = e - j * kW;
    for (int ks = d * kW + w; ks < nks; ks += W)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(A + (size_t)j * K + ks * 16));
  }
  // x_lora may be the output of the grid before this one
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float acc[NJ][4];
#pragma unroll
  for (int jt = 0; jt < NJ; ++jt) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.0f;
  const bool r0 = g < M, r1 = g + 8 < M;
  const T* x0 = X + (size_t)(r0 ? g : 0) * K + 2 * t;
  const T* x1 = X + (size_t)(r1 ? g + 8 : 0) * K + 2 * t;
  for (int ks = d * kW + warp; ks < nks; ks += KB * W) {
    uint32_t a[KB][4], b[KB][NJ][2];
#pragma unroll
    for (int i = 0; i < KB; ++i)
      if (i == 0 || ks + i * W < nks) down_kstep<DT, NJ>(x0, x1, A, K, r, nj, r0, r1, (ks + i * W) * 16, g, t, a[i], b[i]);
#pragma unroll
    for (int i = 0; i < KB; ++i) {
      if (i > 0 && ks + i * W >= nks) break;
#pragma unroll
      for (int jt = 0; jt < NJ; ++jt)
        if (jt < nj) Mma16816<DT>::run(acc[jt], a[i][0], a[i][1], a[i][2], a[i][3], b[i][jt][0], b[i][jt][1]);
    }
  }
  float* red = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int jt = 0; jt < NJ; ++jt) {
    if (jt < nj) {
      float* r_lo = red + (warp * 16 + g) * RP + jt * 8 + 2 * t;
      float* r_hi = red + (warp * 16 + g + 8) * RP + jt * 8 + 2 * t;
      r_lo[0] = acc[jt][0], r_lo[1] = acc[jt][1], r_hi[0] = acc[jt][2], r_hi[1] = acc[jt][3];
    }
  }
  __syncthreads();
  float* part = p.partial + (size_t)d * M * r;
  for (int e = tid; e < M * r; e += kNfBlockThreads) {
    const int m = e / r, j = e - m * r;
    float s = 0.0f;
    for (int w = 0; w < kW; ++w) s += red[(w * 16 + m) * RP + j];
    part[e] = s;
  }
  __syncthreads();  // every partial store of the CTA precedes the release below
  if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.counters) : "memory");
}

// 2-D tiled TMA load of box (x, y) of `map` into shared memory, completing on `bar`
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned, size a multiple of 16), completing on `bar`
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
// barrier of the consumer warps only (the producer warp never joins it)
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kNfThreads) : "memory"); }
// the producer warp's one-time signal that the CTA's mbarriers and flags are
// initialized (it arrives, the consumers wait)
__device__ __forceinline__ void start_arrive() { asm volatile("bar.arrive 2, %0;" ::"n"(kNfBlockThreads) : "memory"); }
__device__ __forceinline__ void start_wait() { asm volatile("bar.sync 2, %0;" ::"n"(kNfBlockThreads) : "memory"); }

// the 16-bit element of `w` at bit 0 / bit 16, widened
template <int DT>
__device__ __forceinline__ float lo16_f32(uint32_t w) {
  if constexpr (DT == RQ_BF16) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
template <int DT>
__device__ __forceinline__ float hi16_f32(uint32_t w) {
  if constexpr (DT == RQ_BF16) return __uint_as_float(w & 0xffff0000u);
  else return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
// acc + a[0]*b[0] + ... + a[7]*b[7] over eight packed 16-bit elements, one
// fused multiply-add per element in element order
template <int DT>
__device__ __forceinline__ float dot8(uint4 a, uint4 b, float acc) {
  const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc = fmaf(lo16_f32<DT>(av[i]), lo16_f32<DT>(bv[i]), acc);
    acc = fmaf(hi16_f32<DT>(av[i]), hi16_f32<DT>(bv[i]), acc);
  }
  return acc;
}

// (a0, a1) += (p0, p1) * s as one packed fp32 FMA (each element rounded
// once, as fmaf would)
__device__ __forceinline__ void fma2(float& a0, float& a1, float p0, float p1, float s) {
  unsigned long long a, pp, ss;
  asm("mov.b64 %0, {%1,%2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1,%2};" : "=l"(pp) : "f"(p0), "f"(p1));
  asm("mov.b64 %0, {%1,%1};" : "=l"(ss) : "f"(s));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(pp), "l"(ss));
  asm("mov.b64 {%0,%1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
}

// The reference's dequantized weight pair, rounded as it rounds it: each
// fp32 level times the fp32 block scale (one fp32 rounding), then to the
// activation dtype (round to nearest even).
template <int DT>
__device__ __forceinline__ uint32_t ref_pair(uint2 lv, float s) {
  unsigned long long t, ss, r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(t) : "r"(lv.x), "r"(lv.y));
  asm("mov.b64 %0, {%1,%1};" : "=l"(ss) : "f"(s));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(t), "l"(ss));
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
  uint32_t d;
  if constexpr (DT == RQ_BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// int8 codes B and B+1 of a code word as a 16-bit pair (exact: |code| <=
// 128), from u = word ^ 0x80808080 (each code + 128, as an unsigned byte),
// without integer-to-float conversions (their pipe is narrow):
//   bf16: the byte under 0x4B00_0000 is the fp32 2^23 + 128 + v; one packed
//         fp32 subtraction of 2^23 + 128 leaves v, one packed convert;
//   f16:  the byte under 0x64 is the half 1024 + 128 + v; one packed half
//         subtraction of 1152 leaves v.
template <int DT, int B>
__device__ __forceinline__ uint32_t i8pair(uint32_t u) {
  uint32_t d;
  if constexpr (DT == RQ_BF16) {
    const uint32_t b0 = __byte_perm(u, 0x4B000000u, 0x7650u | B), b1 = __byte_perm(u, 0x4B000000u, 0x7650u | (B + 1));
    unsigned long long t, r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(t) : "r"(b0), "r"(b1));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(t), "l"(0xCB000080CB000080ull));  // - (2^23 + 128), twice
    float f0, f1;
    asm("mov.b64 {%0,%1}, %2;" : "=f"(f0), "=f"(f1) : "l"(r));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(f1), "f"(f0));
  } else {
    const uint32_t h = __byte_perm(u, 0x64646464u, (uint32_t)B | (4u << 4) | ((uint32_t)(B + 1) << 8) | (4u << 12));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(0x64806480u));  // - 1152, twice
  }
  return d;
}

template <int DT, int MG>
__device__ __forceinline__ void kstep(float (&part)[MG][4], bool first, uint32_t a0, uint32_t a1, uint32_t a2,
                                      uint32_t a3, const uint32_t (&x)[MG][8], int j) {
#pragma unroll
  for (int gr = 0; gr < MG; ++gr) {
    if (first)
      Mma16816Zero<DT>::run(part[gr], a0, a1, a2, a3, x[gr][2 * j], x[gr][2 * j + 1]);
    else
      Mma16816<DT>::run(part[gr], a0, a1, a2, a3, x[gr][2 * j], x[gr][2 * j + 1]);
  }
}

// tile row read by MMA row g (0..7) of a 16-row tile (rows g+8 read it + 8):
// the identity in the 3-D layout, a permutation in the 2-D one
__host__ __device__ __forceinline__ int mma_row(int g, int wide) { return wide ? g : 2 * (g & 3) + (g >> 2); }
// MMA row of tile row rr (0..15) modulo 8
__host__ __device__ __forceinline__ int mma_of_row(int rr, int wide) { return wide ? (rr & 7) : ((rr & 7) >> 1) + 4 * (rr & 1); }

// The block scales of blocks [b0, b0 + W) of a pass's R rows (first row c0)
// into the staged table sc (block b0 at sc row 0), for passes whose table
// is decoded window by window: from the raw bytes in shared memory (the
// tail under 16 bytes from global memory), the second level through the
// fp8 / int8 table times c2_scales.
__device__ __noinline__ void nf4_decode_window(const GemvArgs& p, int wide, int nbk, int esz, int sp, int c0, int R,
                                               int b0, int W, uint32_t inraw, const unsigned char* raw,
                                               const float* sclut, const float* c2s_sm, float* sc) {
  const int tid = threadIdx.x, fmt = p.w.fmt;
  const int64_t f0 = (int64_t)c0 * nbk;
  const int total = R * W, f0lo = (int)(f0 & 255), dq = kNfThreads / W, dr = kNfThreads - dq * W;
  int rl = tid / W, bb = tid - rl * W;
  for (int i = tid; i < total; i += kNfThreads) {
    const int e = rl * nbk + b0 + bb;  // entry of the pass
    float v;
    if (fmt == RQ_W_NF4) {
      if ((uint32_t)e < inraw) v = esz == 4 ? reinterpret_cast<const float*>(raw)[e] : load_scalar(raw, p.w.sdt, e);
      else v = load_scalar(p.w.scales, p.w.sdt, f0 + e);
    } else {
      const uint32_t code = (uint32_t)e < inraw ? (uint32_t)raw[e] : (uint32_t)__ldg(p.w.c2 + f0 + e);
      v = sclut[code] * c2s_sm[(f0lo + e) >> 8];
    }
    const int rr = rl & 15, gg = mma_of_row(rr, wide);
    sc[bb * sp + (rl >> 4) * 16 + gg * 2 + (rr >> 3)] = v;
    bb += dr;
    rl += dq;
    if (bb >= W) bb -= W, ++rl;
  }
}

template <int DT, int MG, int NT, bool EXACT, bool SS, bool WIN, int WK>
__global__ void __launch_bounds__(kNfBlockThreads, 1) gemv_nf4_k(const __grid_constant__ Nf4Args q) {
  using T = typename DType<DT>::T;
  const GemvArgs& p = q.a;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[2 * kNfMaxSlots + 2];  // full[S], empty[S], scales full / empty
  __shared__ int abort_flag, issued, raw_issued, producer_done, stop, gather_skip;
  __shared__ uint32_t gather_epoch;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // The next layer's down-product kernel (a programmatic dependent) may be
  // scheduled beside this grid now: it waits for this grid to finish before
  // it reads anything but weights.
  asm volatile("griddepcontrol.launch_dependents;");
  // The gather's flags and counters are written by the calls before this
  // one: a gather kernel waits for the grids before it at once -- unless it
  // follows the down-product kernel (xsafe), which let it launch only after
  // its own wait, when those calls had finished.
  if (q.a.gather && !q.xsafe) asm volatile("griddepcontrol.wait;" ::: "memory");
  // fused LoRA down product: the grid's first kNfDownCtas CTAs
  if (p.fuse_down && blockIdx.x < (unsigned)kNfDownCtas) {
    if (p.r <= 16) down_role<DT, 2>(p, smem);
    else if (p.r <= 32) down_role<DT, 4>(p, smem);
    else down_role<DT, 8>(p, smem);
    return;
  }
  const int cta = (int)blockIdx.x - (p.fuse_down ? kNfDownCtas : 0);  // GEMV CTA index
  const int N = (int)p.w.N, K = (int)p.w.K, M = (int)p.M;
  const int nbk = K >> 6;
  const int nst = (nbk + kStageBlocks - 1) / kStageBlocks;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t ring = (sbase + q.ring_off + 1023u) & ~1023u;  // shared address (swizzle atoms are 1 KB)
  const int sp = q.sp, S = q.slots;
  const uint32_t slot_bytes = q.slot_bytes;
  constexpr uint32_t kBox = NT * 16 * 128;  // one 128-byte-wide code box
  // code boxes of a stage (NF4: 256 bytes a row, int8: 512) and X after them
  constexpr uint32_t kCodeBoxes = WK ? 4u : 2u, kXOff = kCodeBoxes * kBox;
  const uint32_t full0 = (uint32_t)__cvta_generic_to_shared(bars), empty0 = full0 + kNfMaxSlots * 8;
  const uint32_t scfull = full0 + 2 * kNfMaxSlots * 8, scempty = scfull + 8;
  // raw scale bytes of the pass at rows [c0, c0+R): one copy of the 16-byte
  // aligned part (the rest, under 16 bytes, is read directly)
  const int esz = q.esz;
  const unsigned char* rawsrc = static_cast<const unsigned char*>(
      p.w.fmt == RQ_W_NF4 || p.w.fmt == RQ_W_INT8 ? p.w.scales : (const void*)p.w.c2);
  auto raw_bytes = [&](int R) { return (uint32_t)(R * nbk * esz) & ~15u; };
  volatile int* abortp = &abort_flag;
  volatile int* issuedp = &issued;
  volatile int* raw_issuedp = &raw_issued;
  volatile int* donep = &producer_done;

  const int tb = cta * q.tpc;
  const int te = tb + q.tpc < q.tiles ? tb + q.tpc : q.tiles;
  auto pass_tiles = [&](int ch, int& t0, int& t1) {
    t0 = tb + ch * NT;
    t1 = t0 + NT < te ? t0 + NT : te;
  };

  if (warp == kNfWarps) {
    // ---- producer: initializes the mbarriers and flags itself and starts
    // issuing at once; the consumers wait for its start signal only before
    // their first mbarrier wait (their table builds run meanwhile)
    if (lane == 0) {
      // every kernel parameter the issue path reads, loaded at once: the
      // constant-bank misses overlap instead of following one another
      asm volatile("" ::"r"(q.chunks), "r"(q.tpc), "r"(q.tiles), "r"(q.esz), "r"(q.raw_off), "r"(q.wide), "r"(S),
                   "r"(ring), "r"(slot_bytes), "r"(M), "r"(N), "r"(nbk), "l"(rawsrc));
      asm volatile("prefetch.tensormap [%0];" ::"l"(&q.wmap) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&q.xmap) : "memory");
      for (int i = 0; i < S; ++i) {
        mbar_init(full0 + 8 * i, 1);
        mbar_init(empty0 + 8 * i, SS ? kStageBlocks : kNfWarps);  // the warps that take the stage
      }
      mbar_init(scfull, 1);
      mbar_init(scempty, 1);
      abort_flag = 0;
      issued = 0;
      raw_issued = 0;
      producer_done = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    start_arrive();
    // ---- stage u (over all passes) into slot u % S.  X may be the output
    // of the grid this one overlaps: the first ring fill streams the codes
    // only, and X of those stages follows once the grids before this one
    // have finished (griddepcontrol.wait; gather kernels waited at start).
    if (lane == 0) {
      const uint32_t bytes = kXOff + (uint32_t)M * 1024;
      uint32_t u = 0, xpend = 0;  // stages 0 .. xpend-1 of pass 0 still wait for X
      bool xopen = p.gather != 0 || q.xsafe != 0;
      const uint32_t fill = (uint32_t)(nst < S ? nst : S);
      auto open_x = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (uint32_t v = 0; v < xpend; ++v)
          tma_load_2d(ring + v * slot_bytes + kXOff, &q.xmap, (int)v * 256, 0, full0 + 8 * v);
        xpend = 0;
        xopen = true;
      };
      for (int ch = 0; ch < q.chunks && !*abortp; ++ch) {
        int t0, t1;
        pass_tiles(ch, t0, t1);
        if (t1 <= t0) break;
        // the pass's raw scales first (the buffer is free once the consumers
        // decoded the previous pass's)
        if (ch > 0 && !mbar_wait(scempty, (ch - 1) & 1, abortp)) break;
        const int R = (t1 * 16 < N ? t1 * 16 : N) - t0 * 16;
        const uint32_t rb = raw_bytes(R);
        // with one pass, the pass's rows of LoRA B too (a weight, written
        // before the down-product kernel started; R * r * 2 bytes, a multiple
        // of 16 at a 16-byte aligned source)
        const uint32_t bb = q.bsm ? (uint32_t)(R * p.r * 2) : 0u;
        mbar_expect_tx(scfull, rb + bb);
        if (rb) bulk_load(sbase + q.raw_off, rawsrc + (size_t)t0 * 16 * nbk * esz, rb, scfull);
        if (bb)
          bulk_load(sbase + q.bsm_off, static_cast<const unsigned char*>(p.lora_b) + (size_t)t0 * 16 * p.r * 2, bb,
                    scfull);
        *raw_issuedp = ch + 1;
        for (int s = 0; s < nst; ++s, ++u) {
          const uint32_t slot = u % S;
          if (u >= (uint32_t)S && !mbar_wait(empty0 + 8 * slot, ((u / S) - 1) & 1, abortp)) break;
          const uint32_t dst = ring + slot * slot_bytes, bar = full0 + 8 * slot;
          mbar_expect_tx(bar, bytes);
          if (WK) {  // int8: [rows][4][128 B], 512 bytes a row
            tma_load_3d(dst, &q.wmap, 0, 4 * s, t0 * 16, bar);
          } else if (q.wide) {
            tma_load_3d(dst, &q.wmap, 0, 2 * s, t0 * 16, bar);
          } else {
            tma_load_2d(dst, &q.wmap, s * 256, t0 * 16, bar);
            tma_load_2d(dst + kBox, &q.wmap, s * 256 + 128, t0 * 16, bar);
          }
          if (xopen) {
            tma_load_2d(dst + kXOff, &q.xmap, s * 256, 0, bar);
          } else {
            ++xpend;  // pass 0, stage s == u in slot u
            if (xpend == fill) open_x();
          }
          *issuedp = (int)(u + 1);
        }
      }
      if (xpend) open_x();  // the loop ended early: every issued stage still completes
      __threadfence_block();
      *donep = 1;
    }
    return;
  }

  // ---- consumers
  if (p.gather && warp == 0) {  // announce this rank's entry first thing
    const uint32_t e = gather_epoch_of(p.gth);
    gather_enter(p.gth, e, lane);
    if (lane == 0) gather_epoch = e, gather_skip = 0;
  }
  unsigned char* lut = smem;
  float* sc = reinterpret_cast<float*>(smem + q.sc_off);
  float* sclut = reinterpret_cast<float*>(smem + q.aux_off);
  T* tl = reinterpret_cast<T*>(smem + q.tl_off);
  T* stg = reinterpret_cast<T*>(smem + q.stg_off);
  const uint32_t lanesel = sbase + (uint32_t)(lane * (EXACT ? 8 : 4));
  // warp pair bw = warp % 8 multiplies block bw of each stage; warp bw + 8 h
  // takes the pass's tiles nt = h, h + 2, ...
  const int bw = warp % kStageBlocks, th = warp / kStageBlocks;
  // lane's code bytes in a slot: logical 16-byte chunk 2*(bw & 3) + (t >> 1)
  // of 128-byte half bw >> 2 of tile row mma_row(g) (+16 nt + 8 h), half t & 1;
  // the 128-byte shared rows are swizzled by their index mod 8.
  //   3-D: shared row 2*r + half -> per tile 4096 bytes, per h 2048
  //   2-D: half at kBox, shared row r -> per tile 2048 bytes, per h 1024
  //   int8: the lane's 16 bytes of block bw are 16-byte chunk 4*(bw & 1) + t of
  //   quarter bw >> 1 of the tile row; shared row 4*r + quarter -> per tile
  //   8192 bytes, per h 4096
  const int wide = WK ? 1 : q.wide;
  const int pg = mma_row(g, wide), half = bw >> 2, lch = 2 * (bw & 3) + (t >> 1);
  // (a tile is 16, 32 or 64 shared rows: the swizzle phase repeats per tile)
  const uint32_t tstep = WK ? 8192u : (wide ? 4096u : 2048u), hstep = tstep / 2;
  const uint32_t cofs =
      WK ? (uint32_t)(4 * pg + (bw >> 1)) * 128 + ((((bw & 1) * 4 + t) ^ ((4 * pg + (bw >> 1)) & 7)) << 4)
         : (wide ? (uint32_t)(2 * pg + half) * 128 + (((lch ^ (2 * (pg & 3) + half)) << 4) | ((t & 1) << 3))
                 : (uint32_t)half * kBox + pg * 128 + (((lch ^ pg) << 4) | ((t & 1) << 3)));
  // lane's X in a slot: token gr*8 + g (tokens past M read token M-1, results
  // dropped), columns of block bw, 16 t .. 16 t + 15
  uint32_t xofs[MG];
#pragma unroll
  for (int gr = 0; gr < MG; ++gr) {
    const int m = gr * 8 + g;
    xofs[gr] = kXOff + (uint32_t)(m < M ? m : M - 1) * 1024 + bw * 128 + t * 32;
  }

  // decoded scales of the pass at rows [c0, c0+R) into sc in fragment order
  // [block][tile][MMA row g][g / g+8]
  const int fmt = p.w.fmt;
  const unsigned char* raw = smem + q.raw_off;
  float* c2s_sm = reinterpret_cast<float*>(smem + q.raw_off + ((NT * 16 * nbk * esz + 15) & ~15));
  auto c2s_load = [&](int c0, int R) {  // the pass's c2_scales (one per 256 blocks)
    if (fmt == RQ_W_NF4 || WK) return;
    const int64_t f0 = (int64_t)c0 * nbk;
    const int n = (int)(((f0 + (int64_t)R * nbk - 1) >> 8) - (f0 >> 8)) + 1;
    for (int i = tid; i < n; i += kNfThreads) c2s_sm[i] = __ldg(p.w.c2s + (f0 >> 8) + i);
  };
  auto decode = [&](int c0, int R) {
    const int64_t f0 = (int64_t)c0 * nbk;
    const int total = R * nbk, inraw = (int)(raw_bytes(R) / esz);
    // entry e = rl * nbk + b (row rl of the pass, block b), stepped by
    // kNfThreads without a division per entry; its c2_scales entry is
    // (f0 % 256 + e) / 256 of the pass's
    const int f0lo = (int)(f0 & 255), dq = kNfThreads / nbk, dr = kNfThreads - dq * nbk;
    int rl = tid / nbk, b = tid - rl * nbk;
    auto put = [&](float v) {
      const int rr = rl & 15, gg = mma_of_row(rr, q.wide);
      sc[b * sp + (rl >> 4) * 16 + gg * 2 + (rr >> 3)] = v;
      b += dr;
      rl += dq;
      if (b >= nbk) b -= nbk, ++rl;
    };
    // the entries in the shared copy, then the tail (under 16 bytes) from
    // global memory: separate loops, so that no shared entry waits on a
    // global load the compiler would otherwise issue for every entry
    int e = tid;
    if (fmt == RQ_W_NF4 || fmt == RQ_W_INT8) {
      for (; e < inraw; e += kNfThreads)
        put(esz == 4 ? reinterpret_cast<const float*>(raw)[e] : load_scalar(raw, p.w.sdt, e));
      for (; e < total; e += kNfThreads) put(load_scalar(p.w.scales, p.w.sdt, f0 + e));
    } else {
      // four entries a thread per round, their loads ahead of the stores
      // (four independent load chains instead of one)
      for (; e + 3 * kNfThreads < inraw; e += 4 * kNfThreads) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = sclut[raw[e + i * kNfThreads]] * c2s_sm[(f0lo + e + i * kNfThreads) >> 8];
#pragma unroll
        for (int i = 0; i < 4; ++i) put(v[i]);
      }
      for (; e < inraw; e += kNfThreads) put(sclut[raw[e]] * c2s_sm[(f0lo + e) >> 8]);
      for (; e < total; e += kNfThreads) put(sclut[__ldg(p.w.c2 + f0 + e)] * c2s_sm[(f0lo + e) >> 8]);
    }
  };

  const int swin = q.sw;  // 0: whole pass

  int t0, t1;
  pass_tiles(0, t0, t1);
  if (t1 > t0) c2s_load(t0 * 16, (t1 * 16 < N ? t1 * 16 : N) - t0 * 16);
  // code table (entry v: 32 copies of the pair (T[v & 15], T[v >> 4])) and
  // the second-level table, built while the first stages are in flight
  // (int8 codes need neither)
  if constexpr (WK) {
  } else if constexpr (EXACT) {
    // entry v: 32 copies of the fp32 pair (T[v & 15], T[v >> 4]), 8 bytes a lane
    const float lvl = nf4_level_imm(lane & 15);
#pragma unroll 1
    for (int k = 0; k < 256 * 16 / kNfThreads; ++k) {
      const int v = k * (kNfThreads / 16) + (tid >> 4);
      const uint32_t a = __float_as_uint(__shfl_sync(0xffffffffu, lvl, v & 15));
      const uint32_t b = __float_as_uint(__shfl_sync(0xffffffffu, lvl, v >> 4));
      *reinterpret_cast<uint4*>(lut + v * 256 + (tid & 15) * 16) = make_uint4(a, b, a, b);
    }
  } else {
    const float lvl = nf4_level_imm(lane & 15);
#pragma unroll 1
    for (int k = 0; k < 256 * 8 / kNfThreads; ++k) {
      const int v = k * (kNfThreads / 8) + (tid >> 3);
      const uint32_t w = pack2<DT>(__shfl_sync(0xffffffffu, lvl, v & 15), __shfl_sync(0xffffffffu, lvl, v >> 4));
      *reinterpret_cast<uint4*>(lut + v * 128 + (tid & 7) * 16) = make_uint4(w, w, w, w);
    }
  }
  if (!WK && fmt != RQ_W_NF4 && tid < 256)
    sclut[tid] = fmt == RQ_W_NF4_DQ_FP8 ? e4m3fnuz_to_f32(tid) : ieee_div((float)(int8_t)tid, 127.0f);

  start_wait();  // the producer's mbarriers and flags are initialized
  uint32_t u = 0;       // stages consumed (over all passes)
  uint32_t cslot = 0, cphase = 0;  // u % S and (u / S) & 1, kept without divisions
  uint32_t passes = 0;  // raw-scale copies waited for
  for (int ch = 0; ch < q.chunks; ++ch) {
    if (ch > 0) pass_tiles(ch, t0, t1);
    if (t1 <= t0) break;
    const int ntl = t1 - t0, c0 = t0 * 16;
    const int R = (t1 * 16 < N ? t1 * 16 : N) - c0;
    if (ch > 0) c2s_load(c0, R);
    consumer_sync();  // tables and c2_scales in place
    // the pass's raw scales have landed: decode them, then hand the buffer back
    mbar_wait(scfull, ch & 1, abortp);
    ++passes;
    if constexpr (WIN)
      nf4_decode_window(p, q.wide, nbk, esz, sp, c0, R, 0, swin * kStageBlocks < nbk ? swin * kStageBlocks : nbk,
                        raw_bytes(R) / esz, raw, sclut, c2s_sm, sc);
    else if constexpr (WK != 2)  // int8 per-row scales apply in the epilogue
      decode(c0, R);
    consumer_sync();
    if (tid == 0) mbar_arrive(scempty);

    // stage split: this warp takes stages s = th, th + 2, ... and every tile
    // of the pass; tile split (16-token passes of 4+ tiles, whose
    // accumulators would not fit in registers): every stage, tiles
    // nt = th + 2i
    static_assert(!SS || nf4_stage_split(MG, NT), "stage split holds every tile's accumulators");
    constexpr int NTW = SS ? NT : (NT + kNfSplit - 1) / kNfSplit;
    float acc[NTW][MG][4];
#pragma unroll
    for (int i = 0; i < NTW; ++i)
#pragma unroll
      for (int gr = 0; gr < MG; ++gr) acc[i][gr][0] = acc[i][gr][1] = acc[i][gr][2] = acc[i][gr][3] = 0.0f;
    const float* scw = sc + bw * sp + (SS ? 0 : th * 16) + g * 2;
    const uint32_t cofs_w = cofs + (SS ? 0u : th * tstep);

    // stages [s_begin, s_end) against the scale table of the window that
    // starts at stage s0
    auto run_stages = [&](int s_begin, int s_end, int s0) {
    for (int s = s_begin; s < s_end; ++s, ++u) {
      const uint32_t slot = cslot, par = cphase;
      if (++cslot == (uint32_t)S) cslot = 0, cphase ^= 1u;
      if (SS && (s & (kNfSplit - 1)) != th) continue;
      const bool ok = mbar_wait(full0 + 8 * slot, par, abortp);
      const int b = s * kStageBlocks + bw;
      if (ok && b < nbk) {
        const uint32_t sl = ring + slot * slot_bytes;
        uint32_t x[MG][8];
#pragma unroll
        for (int gr = 0; gr < MG; ++gr) {
          uint4 u0, u1;
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(u0.x), "=r"(u0.y), "=r"(u0.z), "=r"(u0.w) : "r"(sl + xofs[gr]));
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(u1.x), "=r"(u1.y), "=r"(u1.z), "=r"(u1.w) : "r"(sl + xofs[gr] + 16));
          x[gr][0] = u0.x, x[gr][1] = u0.y, x[gr][2] = u0.z, x[gr][3] = u0.w;
          x[gr][4] = u1.x, x[gr][5] = u1.y, x[gr][6] = u1.z, x[gr][7] = u1.w;
        }
        const float* sb = scw + (size_t)(s - s0) * kStageBlocks * sp;
#pragma unroll
        for (int i = 0; i < NTW; ++i) {
          constexpr int kStep = SS ? 1 : kNfSplit;  // tile stride of this warp's tiles
          if (!SS && NT % kNfSplit != 0 && th + kNfSplit * i >= NT) break;
          if constexpr (WK != 0) {
            // int8: 16 codes of row g and of row g+8; word j holds the codes
            // of k-step j (k 4j .. 4j+3 of the lane's 16, as X is laid out)
            uint4 l4, h4;
            asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(l4.x), "=r"(l4.y), "=r"(l4.z), "=r"(l4.w)
                         : "r"(sl + cofs_w + i * kStep * tstep));
            asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(h4.x), "=r"(h4.y), "=r"(h4.z), "=r"(h4.w)
                         : "r"(sl + cofs_w + i * kStep * tstep + hstep));
            // codes + 128 as unsigned bytes (i8pair)
            const uint32_t lw[4] = {l4.x ^ 0x80808080u, l4.y ^ 0x80808080u, l4.z ^ 0x80808080u, l4.w ^ 0x80808080u};
            const uint32_t hw[4] = {h4.x ^ 0x80808080u, h4.y ^ 0x80808080u, h4.z ^ 0x80808080u, h4.w ^ 0x80808080u};
            if constexpr (WK == 2) {
              // per-row scales: the codes multiply straight into the
              // accumulators, the row scale applies in the epilogue
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t a0 = i8pair<DT, 0>(lw[j]), a1 = i8pair<DT, 0>(hw[j]);
                const uint32_t a2 = i8pair<DT, 2>(lw[j]), a3 = i8pair<DT, 2>(hw[j]);
#pragma unroll
                for (int gr = 0; gr < MG; ++gr)
                  Mma16816<DT>::run(acc[i][gr], a0, a1, a2, a3, x[gr][2 * j], x[gr][2 * j + 1]);
              }
            } else {
              const float2 sv = *reinterpret_cast<const float2*>(sb + i * kStep * 16);
              float part[MG][4];
#pragma unroll
              for (int j = 0; j < 4; ++j)
                kstep<DT, MG>(part, j == 0, i8pair<DT, 0>(lw[j]), i8pair<DT, 0>(hw[j]), i8pair<DT, 2>(lw[j]),
                              i8pair<DT, 2>(hw[j]), x, j);
#pragma unroll
              for (int gr = 0; gr < MG; ++gr) {
                fma2(acc[i][gr][0], acc[i][gr][1], part[gr][0], part[gr][1], sv.x);
                fma2(acc[i][gr][2], acc[i][gr][3], part[gr][2], part[gr][3], sv.y);
              }
            }
            continue;
          }
          uint2 lo, hi;
          asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(lo.x), "=r"(lo.y) : "r"(sl + cofs_w + i * kStep * tstep));
          asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];"
                       : "=r"(hi.x), "=r"(hi.y)
                       : "r"(sl + cofs_w + i * kStep * tstep + hstep));
          const float2 sv = *reinterpret_cast<const float2*>(sb + i * kStep * 16);
          float part[MG][4];
          if constexpr (EXACT) {
            // the reference's weights (level x scale, rounded), multiplied
            // straight into the accumulators: no per-block scale step
            const float sg = sv.x, sg8 = sv.y;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t wlo = j < 2 ? lo.x : lo.y, whi = j < 2 ? hi.x : hi.y;
              const uint2 l0 = (j & 1) ? lut4<2>(wlo, lanesel) : lut4<0>(wlo, lanesel);
              const uint2 h0 = (j & 1) ? lut4<2>(whi, lanesel) : lut4<0>(whi, lanesel);
              const uint2 l1 = (j & 1) ? lut4<3>(wlo, lanesel) : lut4<1>(wlo, lanesel);
              const uint2 h1 = (j & 1) ? lut4<3>(whi, lanesel) : lut4<1>(whi, lanesel);
              const uint32_t a0 = ref_pair<DT>(l0, sg), a1 = ref_pair<DT>(h0, sg8);
              const uint32_t a2 = ref_pair<DT>(l1, sg), a3 = ref_pair<DT>(h1, sg8);
#pragma unroll
              for (int gr = 0; gr < MG; ++gr) Mma16816<DT>::run(acc[i][gr], a0, a1, a2, a3, x[gr][2 * j], x[gr][2 * j + 1]);
            }
            (void)part;
            continue;
          } else {
            kstep<DT, MG>(part, true, lut2<0>(lo.x, lanesel), lut2<0>(hi.x, lanesel), lut2<1>(lo.x, lanesel),
                          lut2<1>(hi.x, lanesel), x, 0);
            kstep<DT, MG>(part, false, lut2<2>(lo.x, lanesel), lut2<2>(hi.x, lanesel), lut2<3>(lo.x, lanesel),
                          lut2<3>(hi.x, lanesel), x, 1);
            kstep<DT, MG>(part, false, lut2<0>(lo.y, lanesel), lut2<0>(hi.y, lanesel), lut2<1>(lo.y, lanesel),
                          lut2<1>(hi.y, lanesel), x, 2);
            kstep<DT, MG>(part, false, lut2<2>(lo.y, lanesel), lut2<2>(hi.y, lanesel), lut2<3>(lo.y, lanesel),
                          lut2<3>(hi.y, lanesel), x, 3);
          }
#pragma unroll
          for (int gr = 0; gr < MG; ++gr) {
            fma2(acc[i][gr][0], acc[i][gr][1], part[gr][0], part[gr][1], sv.x);
            fma2(acc[i][gr][2], acc[i][gr][3], part[gr][2], part[gr][3], sv.y);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * slot);  // this warp is done with the slot
    }
    };
    if constexpr (WIN) {
      for (int s0 = 0; s0 < nst; s0 += swin) {
        if (s0 > 0) {
          // next scale window: every warp is done with the stages before s0
          consumer_sync();
          const int b0 = s0 * kStageBlocks;
          nf4_decode_window(p, q.wide, nbk, esz, sp, c0, R, b0,
                            nbk - b0 < swin * kStageBlocks ? nbk - b0 : swin * kStageBlocks, raw_bytes(R) / esz, raw,
                            sclut, c2s_sm, sc);
          consumer_sync();
        }
        run_stages(s0, s0 + swin < nst ? s0 + swin : nst, s0);
      }
    } else {
      run_stages(0, nst, 0);
    }

    consumer_sync();  // every warp is done with the ring (the partial sums may reuse it)
    if (tid == 0) stop = *abortp;  // one decision for all consumers (the producer may set the flag any time)
    consumer_sync();
    if (stop) break;
    float* red = q.red_off ? reinterpret_cast<float*>(smem + q.red_off) : reinterpret_cast<float*>(smem + (ring - sbase));
    float4* red4 = reinterpret_cast<float4*>(red);
    // partial sums [part][tile][group][fragment]: stage split, part = warp
    // (every warp holds every tile); tile split, part = block column (the
    // two warps of a column fill disjoint tiles)
#pragma unroll
    for (int i = 0; i < NTW; ++i) {
      const int nt = SS ? i : th + kNfSplit * i;
      if (!SS && NT % kNfSplit != 0 && nt >= NT) break;
#pragma unroll
      for (int gr = 0; gr < MG; ++gr)
        red4[(((SS ? warp : bw) * NT + nt) * MG + gr) * 32 + lane] =
            make_float4(acc[i][gr][0], acc[i][gr][1], acc[i][gr][2], acc[i][gr][3]);
    }
    if (ch == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");  // x.A^T of the kernel before
      if (p.fuse_down) {  // x.A^T from the partials of this grid's down CTAs
        if (tid == 0 && !count_wait(p.counters, kNfDownCtas)) *abortp = 1;
        consumer_sync();
        for (int e = tid; e < M * p.r; e += kNfThreads) {
          float sum = 0.0f;
#pragma unroll
          for (int c = 0; c < kNfDownCtas; ++c) sum += __ldcg(p.partial + (size_t)c * M * p.r + e);
          tl[e] = DType<DT>::from_f32(sum);
        }
      } else if (p.r > 0) {
        const T* td = static_cast<const T*>(p.tdown);
        for (int e = tid; e < M * p.r; e += kNfThreads) tl[e] = td[e];
      }
      // every rank has entered this call before any of its Y is written
      if (p.gather && warp == kNfWarps - 1 && !gather_entered(p.gth, gather_epoch, lane) && lane == 0)
        gather_skip = 1;
    }
    consumer_sync();

    // fragment element e of (tile nt, group gr): lane (g,t) = (e >> 2) & 31,
    // MMA row g + 8 (e >> 1 & 1), token 8 gr + 2t + (e & 1)
    const bool has_bias = p.bias != nullptr, has_lora = p.r > 0;
    const T* lb = static_cast<const T*>(p.lora_b);
    // rows of B and of x.A^T (shared, 16-byte aligned) in 16-byte pieces
    const bool lora_vec = p.r % 8 == 0 && ((uintptr_t)lb % 16) == 0;
    T* y = static_cast<T*>(p.y);
    for (int e = tid; e < NT * MG * 128; e += kNfThreads) {
      const int nt = e / (MG * 128), gr = (e >> 7) % MG, ln = (e >> 2) & 31;
      const int rl = nt * 16 + mma_row(ln >> 2, wide) + ((e >> 1) & 1) * 8, m = gr * 8 + (ln & 3) * 2 + (e & 1);
      if (nt >= ntl || rl >= R || m >= M) continue;
      float sum = 0.0f;
#pragma unroll
      for (int w = 0; w < (SS ? kNfWarps : kStageBlocks); ++w) sum += red[w * (NT * MG * 128) + e];
      const int row = c0 + rl;
      if constexpr (WK == 2) sum *= load_scalar(p.w.scales, p.w.sdt, row);  // int8 per-row scale
      float uu = 0.0f;
      if (has_lora) {
        const T* brow = lb + (size_t)row * p.r;
        const T* trow = tl + m * p.r;
        if (q.bsm) {  // B's rows in shared memory (landed with the raw scales)
          const T* bs = reinterpret_cast<const T*>(smem + q.bsm_off) + (size_t)rl * p.r;
          for (int j = 0; j < p.r; j += 8)
            uu = dot8<DT>(*reinterpret_cast<const uint4*>(trow + j), *reinterpret_cast<const uint4*>(bs + j), uu);
        } else if (lora_vec) {  // 16-byte loads, the same summation order
          for (int j = 0; j < p.r; j += 8)
            uu = dot8<DT>(*reinterpret_cast<const uint4*>(trow + j), __ldg(reinterpret_cast<const uint4*>(brow + j)),
                          uu);
        } else {
#pragma unroll 8
          for (int j = 0; j < p.r; ++j) uu = fmaf(DType<DT>::to_f32(trow[j]), DType<DT>::to_f32(__ldg(brow + j)), uu);
        }
      }
      const float bv = has_bias ? load_scalar(p.bias, p.bdt, row) : 0.0f;
      const T v = DType<DT>::from_f32(lora_epilogue<DT>(sum, has_bias, bv, uu, has_lora, p.s));
      if (p.gather)
        stg[m * (NT * 16) + rl] = v;
      else
        y[(size_t)m * N + row] = v;
    }
    if (p.gather) {
      // the pass's outputs into every rank's Y[:, col + c0 ...]: 16-byte row
      // pieces where the destinations are 16-byte aligned (one NVLink write
      // each), the rest element by element (nothing if a rank never entered
      // the call: the output is then incomplete and the error flag is set)
      consumer_sync();
      if (!gather_skip) {
        const int64_t ld = p.gth.ld, col0 = p.gth.col + c0;
        const int R8 = ((ld | col0) & 7) == 0 ? (R & ~7) : 0, nb8 = R8 / 8;
        for (int i = tid; i < M * nb8; i += kNfThreads) {
          const int m = i / nb8, j = (i - m * nb8) * 8;
          const uint4 v = *reinterpret_cast<const uint4*>(stg + m * (NT * 16) + j);
          const size_t o = (size_t)m * ld + col0 + j;
          for (int rq = 0; rq < p.gth.world; ++rq) *reinterpret_cast<uint4*>(static_cast<T*>(p.gth.outs[rq]) + o) = v;
        }
        const int rest = R - R8;
        for (int i = tid; i < M * rest; i += kNfThreads) {
          const int m = i / rest, j = R8 + (i - m * rest);
          const T v = stg[m * (NT * 16) + j];
          const size_t o = (size_t)m * ld + col0 + j;
          for (int rq = 0; rq < p.gth.world; ++rq) static_cast<T*>(p.gth.outs[rq])[o] = v;
        }
      }
    }
    consumer_sync();  // partial sums (and per-pass scales) are reused by the next pass
  }

  if (*abortp && tid == 0) {
    // a wait gave up: let every issued copy land (bounded) before the CTA's
    // shared memory is released
    for (uint32_t i = 0; i < kWaitLimit && !*donep; ++i) {
    }
    const uint32_t n = (uint32_t)*issuedp, nr = (uint32_t)*raw_issuedp;
    for (uint32_t v = u; v < n; ++v)
      for (uint32_t i = 0; i < kWaitLimit && !mbar_test(full0 + 8 * (v % S), (v / S) & 1); ++i) {
      }
    for (uint32_t v = passes; v < nr; ++v)
      for (uint32_t i = 0; i < kWaitLimit && !mbar_test(scfull, v & 1); ++i) {
      }
  }
  if (p.fuse_down && tid == 0) {
    // the last GEMV CTA zeroes the counters once every GEMV CTA has read the
    // partials (each arrives after its epilogue; an aborted CTA arrives too)
    // and every down CTA has added its arrival
    __threadfence();
    if (atomicAdd(p.counters + 2, 1u) == gridDim.x - kNfDownCtas - 1u) {
      count_wait(p.counters, kNfDownCtas);
      p.counters[2] = 0u;
      p.counters[0] = 0u;
    }
  }
  if (p.gather) {
    // every consumer's stores of the call are ordered before the arrival by
    // the barrier; the arrival's release covers them
    consumer_sync();
    if (warp == 0) gather_arrive(p.gth, lane);
  }
}

// ---------------------------------------------------------------- host side

static size_t align16(size_t v) { return (v + 15) / 16 * 16; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda itself).
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 2-D / 3-D tensor maps, cached by (address, element type, extents, box, swizzle):
// those determine the map completely.
struct MapKey {
  const void* ptr;
  int type, swz, rank;
  uint64_t d[3], stride[2];
  uint32_t box[3];
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && type == o.type && swz == o.swz && rank == o.rank && d[0] == o.d[0] && d[1] == o.d[1] &&
           d[2] == o.d[2] && stride[0] == o.stride[0] && stride[1] == o.stride[1] && box[0] == o.box[0] &&
           box[1] == o.box[1] && box[2] == o.box[2];
  }
};

static int tensor_map(const MapKey& k, CUtensorMap* out) {
  static std::mutex mu;
  static std::vector<std::pair<MapKey, CUtensorMap>> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (const auto& e : cache)
      if (e.first == k) {
        *out = e.second;
        return RQ_OK;
      }
  }
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return RQ_ERR_CUDA;
  const cuuint64_t dims[3] = {k.d[0], k.d[1], k.d[2]}, strides[2] = {k.stride[0], k.stride[1]};
  const cuuint32_t box[3] = {k.box[0], k.box[1], k.box[2]}, es[3] = {1, 1, 1};
  CUtensorMap m;
  auto encode = [&] {
    return enc(&m, (CUtensorMapDataType)k.type, (cuuint32_t)k.rank, const_cast<void*>(k.ptr), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)k.swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    // a thread that has only used the runtime API (autograd's backward
    // thread, for one) may have no driver context bound yet: bind the
    // current device's primary context, as every runtime call on it would,
    // and encode again
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  if (r != CUDA_SUCCESS) {
    set_cuda_error((cudaError_t)(kDriverErrorBase + (int)r));
    return RQ_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 4096) cache.clear();
  cache.emplace_back(k, m);
  *out = m;
  return RQ_OK;
}

// Tensor map for other kernels of the library (cached like the GEMV's).
int tensor_map_encode(int type, int swz, int rank, const void* ptr, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box, CUtensorMap* out) {
  MapKey k{ptr, type, swz, rank, {dims[0], dims[1], dims[2]}, {strides[0], strides[1]}, {box[0], box[1], box[2]}};
  return tensor_map(k, out);
}

struct Nf4Plan {
  int grid, tiles, tpc, chunks, nt, mg, sp, esz, slots, sw, wk;
  size_t smem;
  uint32_t slot_bytes, ring_off, red_off, sc_off, raw_off, aux_off, tl_off, stg_off, bsm_off;
};

// [code table | scales | raw scales + c2_scales of a pass | second-level
// table | x.A^T | staged outputs | ring (1 KB aligned) | partial sums];
// with one pass the partial sums reuse the ring.
static size_t nf4_layout(Nf4Plan* pl, int64_t nbk, int64_t M, int r, bool exact) {
  pl->slot_bytes = (uint32_t)((pl->wk ? 4 : 2) * pl->nt * 16 * 128 + M * 1024);
  size_t off = pl->wk ? 0 : lut_bytes(exact);  // int8 codes need no table
  pl->sc_off = (uint32_t)off;
  int64_t scb = pl->sw && pl->sw * kStageBlocks < nbk ? pl->sw * kStageBlocks : nbk;  // blocks in sc
  if (pl->wk == 2) scb = 0;  // per-row scales
  off += align16((size_t)scb * pl->sp * 4);
  pl->raw_off = (uint32_t)off;
  off += align16((size_t)pl->nt * 16 * nbk * pl->esz) + align16(((size_t)pl->nt * 16 * nbk / 256 + 2) * 4);
  pl->aux_off = (uint32_t)off;
  off += 1024;
  pl->tl_off = (uint32_t)off;
  off += align16((size_t)M * (r > 0 ? r : 0) * 2);
  pl->stg_off = (uint32_t)off;
  off += align16((size_t)M * pl->nt * 16 * 2);
  pl->bsm_off = (uint32_t)off;
  off += align16((size_t)pl->nt * 16 * (r > 0 ? r : 0) * 2);
  pl->ring_off = (uint32_t)off;
  off += 1024;  // room to round the ring up to a 1 KB shared address
  const size_t ring = (size_t)pl->slots * pl->slot_bytes, red = (size_t)(nf4_stage_split(pl->mg, pl->nt) ? kNfWarps : kStageBlocks) * pl->nt * pl->mg * 512;
  if (pl->chunks == 1) {
    pl->red_off = 0;
    pl->smem = off + (ring > red ? ring : red);
  } else {
    pl->red_off = (uint32_t)(off + ring);
    pl->smem = off + ring + red;
  }
  return pl->smem;
}

static bool nf4_plan(int64_t N, int64_t K, int64_t M, int r, int esz, int wk, bool beside, bool exact,
                     Nf4Plan* pl) {
  pl->mg = M > 8 ? 2 : 1;
  pl->esz = esz;
  pl->wk = wk;
  const int64_t tiles = (N + 15) / 16;
  // with the down product running beside it, leave the SMs its cluster uses
  int64_t G = num_sms() - (beside ? kLoraDownCtas : 0);
  if (G > tiles) G = tiles;
  if (G < 1) G = 1;
  const int64_t per = (tiles + G - 1) / G;
  const int64_t nbk = K / 64, nst = (nbk + kStageBlocks - 1) / kStageBlocks;
  const int ntmax = pl->mg == 1 ? kNfMaxNT1 : kNfMaxNT2;
  pl->tiles = (int)tiles;
  for (int64_t ch = (per + ntmax - 1) / ntmax;; ++ch) {
    const int64_t nt = (per + ch - 1) / ch;
    pl->chunks = (int)ch;
    pl->nt = (int)nt;
    pl->tpc = (int)(nt * ch);
    pl->grid = (int)((tiles + pl->tpc - 1) / pl->tpc);
    // deepest ring that fits (at least 2 stages) with the pass's whole
    // scale table; where none fits, with the table decoded 8 stages at a
    // time rather than more passes (default numerics; measured: windows
    // cost more than a few extra ring stages gain, but less than a pass)
    pl->sp = (int)(nt * 16 + 2);
    const int top = (int)(nst < kNfMaxSlots ? (nst > 2 ? nst : 2) : kNfMaxSlots);
    for (int sw : {0, 8}) {
      if (sw && (exact || wk || nst <= sw)) break;  // windows: NF4, default numerics only
      pl->sw = sw;
      for (int s = top; s >= 2; --s) {
        pl->slots = s;
        if (nf4_layout(pl, nbk, M, r, exact) <= kNfSmemMax) return true;
      }
    }
    if (nt == 1) return false;
  }
}

// bytes per raw scale entry of the weight's format (0: per-row scales,
// applied in the epilogue)
static int nf4_esz(const QWeight& w) {
  if (w.fmt == RQ_W_INT8_ROW) return 0;
  if (w.fmt == RQ_W_NF4 || w.fmt == RQ_W_INT8) return w.sdt == RQ_F32 ? 4 : 2;
  return 1;  // c2 codes
}
// kernel code format: 0 NF4 (plain or double-quantized scales), 1 int8
// blockwise, 2 int8 per-row
static int nf4_wk(const QWeight& w) { return w.fmt == RQ_W_INT8 ? 1 : (w.fmt == RQ_W_INT8_ROW ? 2 : 0); }

// Decode numerics: 0 = levels rounded once to the activation dtype, the
// block scale applied to each 64-wide fp32 partial (the default); 1 = the
// reference's weights, level x scale rounded per weight (exact mode).
// RQ_DECODE_EXACT=1 in the environment selects 1 at the first call;
// rq_set_decode_exact() changes it at any time.
static std::atomic<int> g_decode_exact{-1};

bool decode_exact() {
  int v = g_decode_exact.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("RQ_DECODE_EXACT");
    v = (e && e[0] == '1') ? 1 : 0;
    int expected = -1;
    if (!g_decode_exact.compare_exchange_strong(expected, v)) v = expected;
  }
  return v == 1;
}

void set_decode_exact(int on) { g_decode_exact.store(on ? 1 : 0); }

bool gemv_nf4_fits(const QWeight& w, int64_t M, int r) {
  Nf4Plan pl;
  const int wk = nf4_wk(w);
  // the raw scale copy reads 16-byte aligned sources; int8 rows travel as
  // 3-D boxes of 128-byte pieces
  const void* sp = w.fmt == RQ_W_NF4 || w.fmt == RQ_W_INT8 ? w.scales : (const void*)w.c2;
  if (wk != 2 && ((uintptr_t)sp % 16) != 0) return false;
  if (wk && w.K % 128 != 0) return false;
  const bool exact = decode_exact() && wk == 0;
  return encode_tiled() != nullptr && nf4_plan(w.N, w.K, M, r, nf4_esz(w), wk, false, exact, &pl) &&
         nf4_plan(w.N, w.K, M, r, nf4_esz(w), wk, true, exact, &pl);
}

template <int DT, int MG, int NT, bool EXACT, bool SS, bool WIN, int WK>
static int nf4_launch1(const Nf4Args& q, size_t smem, cudaStream_t st) {
  auto kern = gemv_nf4_k<DT, MG, NT, EXACT, SS, WIN, WK>;
  const int rc = ensure_smem_limit((const void*)kern, smem);
  if (rc != RQ_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)q.a.grid);
  cfg.blockDim = dim3(kNfBlockThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;  // X and x.A^T are read only after griddepcontrol.wait
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, q);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  return check_launch();
}

template <int DT, int MG, int NT, int WK>
static int nf4_launch_ss(const Nf4Args& q, size_t smem, cudaStream_t st) {
  if constexpr (nf4_stage_split(MG, NT))
    if (q.stage_split) return nf4_launch1<DT, MG, NT, false, true, false, WK>(q, smem, st);
  return nf4_launch1<DT, MG, NT, false, false, false, WK>(q, smem, st);
}

template <int DT, int MG, int NT, bool EXACT>
static int nf4_launch(const Nf4Args& q, size_t smem, cudaStream_t st) {
  // int8 codes (default numerics, no scale windows)
  if constexpr (!EXACT) {
    if (q.wk == 1) return nf4_launch_ss<DT, MG, NT, 1>(q, smem, st);
    if (q.wk == 2) return nf4_launch_ss<DT, MG, NT, 2>(q, smem, st);
  }
  // scale windows: default numerics, tile split (the plan asks for them
  // only where the whole-pass table leaves a short ring)
  if constexpr (!EXACT)
    if (q.sw) return nf4_launch1<DT, MG, NT, false, false, true, 0>(q, smem, st);
  if constexpr (nf4_stage_split(MG, NT))
    if (q.stage_split) return nf4_launch1<DT, MG, NT, EXACT, true, false, 0>(q, smem, st);
  return nf4_launch1<DT, MG, NT, EXACT, false, false, 0>(q, smem, st);
}

template <int DT, int MG, bool EXACT>
static int nf4_nt(const Nf4Args& q, int nt, size_t smem, cudaStream_t st) {
  switch (nt) {
    case 1: return nf4_launch<DT, MG, 1, EXACT>(q, smem, st);
    case 2: return nf4_launch<DT, MG, 2, EXACT>(q, smem, st);
    case 3: return nf4_launch<DT, MG, 3, EXACT>(q, smem, st);
    case 4: return nf4_launch<DT, MG, 4, EXACT>(q, smem, st);
    case 5: return nf4_launch<DT, MG, 5, EXACT>(q, smem, st);
  }
  if constexpr (MG == 1)
    if (nt == 6) return nf4_launch<DT, MG, 6, EXACT>(q, smem, st);
  return RQ_ERR_INVALID;
}

template <int DT, bool EXACT>
static int nf4_dispatch(const Nf4Args& q, const Nf4Plan& pl, cudaStream_t st) {
  return pl.mg == 2 ? nf4_nt<DT, 2, EXACT>(q, pl.nt, pl.smem, st) : nf4_nt<DT, 1, EXACT>(q, pl.nt, pl.smem, st);
}

int gemv_nf4_forward(const GemvArgs& g, bool beside, cudaStream_t st) {
  if (g.w.K % 64 || ((uintptr_t)g.w.q % 16) || ((uintptr_t)g.x % 16)) return RQ_ERR_ALIGN;
  Nf4Plan pl;
  const int wk = nf4_wk(g.w);
  if (wk && g.w.K % 128) return RQ_ERR_ALIGN;
  const bool exact = decode_exact() && wk == 0;  // the numerics switch is NF4's
  if (!nf4_plan(g.w.N, g.w.K, g.M, g.r, nf4_esz(g.w), wk, beside, exact, &pl)) return RQ_ERR_INVALID;
  Nf4Args q;
  // codes with 128-byte swizzle: NF4 3-D [N][K/256][128] bytes, box 128 x 2 x
  // NT*16 when K % 256 == 0, else 2-D [N][K/2] bytes, box 128 x NT*16; int8
  // 3-D [N][K/128][128] bytes, box 128 x 4 x NT*16;
  // X: 32-bit element pairs [M rows][K/2], box 256 x M
  const uint64_t rowb = (uint64_t)(g.w.K / 2), rows = (uint64_t)g.w.N, nt16 = (uint64_t)(pl.nt * 16);
  q.wide = wk ? 1 : g.w.K % 256 == 0;
  int rc = wk ? tensor_map({g.w.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B, 3,
                            {128, (uint64_t)g.w.K / 128, rows}, {128, (uint64_t)g.w.K}, {128u, 4u, (uint32_t)nt16}},
                           &q.wmap)
          : q.wide ? tensor_map({g.w.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B, 3,
                                 {128, rowb / 128, rows}, {128, rowb}, {128u, 2u, (uint32_t)nt16}},
                                &q.wmap)
                   : tensor_map({g.w.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B, 2,
                                 {rowb, rows, 1}, {rowb, 0}, {128u, (uint32_t)nt16, 1u}},
                                &q.wmap);
  if (rc == RQ_OK)
    rc = tensor_map({g.x, CU_TENSOR_MAP_DATA_TYPE_UINT32, CU_TENSOR_MAP_SWIZZLE_NONE, 2,
                     {rowb, (uint64_t)g.M, 1}, {(uint64_t)(g.w.K * 2), 0}, {256u, (uint32_t)g.M, 1u}},
                    &q.xmap);
  if (rc != RQ_OK) return rc;
  q.a = g;
  q.a.grid = pl.grid + (g.fuse_down ? kNfDownCtas : 0);
  q.tiles = pl.tiles;
  q.tpc = pl.tpc;
  q.chunks = pl.chunks;
  q.sp = pl.sp;
  q.esz = pl.esz;
  q.slots = pl.slots;
  q.sw = pl.sw;
  q.wk = wk;
  q.slot_bytes = pl.slot_bytes;
  q.ring_off = pl.ring_off;
  q.red_off = pl.red_off;
  q.sc_off = pl.sc_off;
  q.raw_off = pl.raw_off;
  q.aux_off = pl.aux_off;
  q.tl_off = pl.tl_off;
  q.stg_off = pl.stg_off;
  q.bsm_off = pl.bsm_off;
  q.bsm = pl.chunks == 1 && g.r > 0 && g.r % 8 == 0 && ((uintptr_t)g.lora_b % 16) == 0;
  // the stage split keeps two stages in consumption at once: only with a
  // ring of 4 or more stages (else nothing would stream meanwhile)
  q.stage_split = nf4_stage_split(pl.mg, pl.nt) && pl.slots >= 4 && pl.sw == 0;
  // behind a separate down-product kernel X is complete at launch; with the
  // down product fused, the grid before may still be writing X
  q.xsafe = g.r > 0 && !g.fuse_down;
  if (g.fuse_down && down_smem(g.r) > pl.smem) pl.smem = down_smem(g.r);
  if (g.xdt == RQ_BF16)
    return exact ? nf4_dispatch<RQ_BF16, true>(q, pl, st) : nf4_dispatch<RQ_BF16, false>(q, pl, st);
  return exact ? nf4_dispatch<RQ_F16, true>(q, pl, st) : nf4_dispatch<RQ_F16, false>(q, pl, st);
}

}  // namespace rq

namespace rq {
int gemm_take_timeouts(unsigned int* v);  // gemm_tcgen05.cu
}

extern "C" int rq_take_kernel_timeouts(unsigned int* count) {
  unsigned int v = 0, w = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, rq::g_kernel_timeouts, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(rq::g_kernel_timeouts, &zero, sizeof(zero));
  if (e != cudaSuccess) {
    rq::set_cuda_error(e);
    return RQ_ERR_CUDA;
  }
  const int rc = rq::gemm_take_timeouts(&w);
  if (rc != RQ_OK) return rc;
  if (count) *count = v + w;
  return RQ_OK;
}
