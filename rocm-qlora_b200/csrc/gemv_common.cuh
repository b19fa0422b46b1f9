// gemv_common.cuh -- pieces shared by the decode GEMV kernels (NF4 streaming
// kernel in gemv_nf4.cu, INT8 kernel in gemv_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include "linear_common.cuh"

namespace rq {

template <int DT> struct Mma16816;
template <> struct Mma16816<RQ_BF16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct Mma16816<RQ_F16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kLoraDownCtas = 8;  // CTAs of the small-M down-product kernel (lora_kernels.cu)
constexpr int kGemvMaxNT = 8;     // 8-row tiles held per warp at most (64 rows)

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
  int grid;
  int tiles;           // ceil(N / 8)
  int chunks;          // row chunks per CTA
  int xdt;             // activation dtype (RQ_BF16 / RQ_F16)
  int gather;          // nonzero: output into every rank's Y per gth (NF4 kernel only)
  RqGather gth;
  // LoRA down product fused into the NF4 GEMV's grid (fuse_down != 0): the
  // grid's first kNfDownCtas CTAs write the partial sums of lora_x . lora_a^T
  int fuse_down;
  const void* lora_x;  // [M, K]
  const void* lora_a;  // [r, K]
  float* partial;      // [kNfDownCtas][M][r] fp32 (workspace)
  unsigned* counters;  // workspace counter area: [0] down CTAs done, [2] GEMV CTAs done
};

constexpr int kNfDownCtas = 8;  // CTAs of the fused down product

// mma.sync m16n8k16 with a zero accumulator input (starts a block partial)
template <int DT> struct Mma16816Zero;
template <> struct Mma16816Zero<RQ_BF16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
  }
};
template <> struct Mma16816Zero<RQ_F16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
  }
};

// Table entry of the code byte found at bit SH of `word`, for this lane.
// The table holds 32 copies interleaved per byte value (entry v, copy l at
// word v*32 + l), so lane l reads bank l: one byte extract (prmt) and one
// indexed shared load.
template <int SH>
__device__ __forceinline__ uint32_t lut_at(uint32_t word, const uint32_t* lut_lane) {
  const uint32_t v = __byte_perm(word, 0u, 0x4440u | (SH / 8));
  return lut_lane[v << 5];
}


// SMs of the current device (cached per device).
inline int num_sms() {
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

constexpr size_t kGemvSmemCap = 113 * 1024;  // two CTAs per SM

// NF4-family GEMV (gemv_nf4.cu): whether a shape fits its shared memory, and
// the launch (grid and tiling chosen inside; always a programmatic launch;
// `beside`: the LoRA down-product kernel runs beside it, so the grid leaves
// that kernel's SMs free).
bool gemv_nf4_fits(const QWeight& w, int64_t M, int r);
// decode numerics (rq_set_decode_exact)
bool decode_exact();
void set_decode_exact(int on);
int gemv_nf4_forward(const GemvArgs& g, bool beside, cudaStream_t st);

}  // namespace rq
