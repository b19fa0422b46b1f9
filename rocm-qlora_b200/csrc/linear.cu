// linear.cu -- host-side dispatch of the QuantLinear+LoRA layer.
//
// Exactly one kernel family runs per call (chosen from shape and dtype):
//   * decode GEMV (gemv_kernels.cu)  M <= 16, bf16/f16 activations, K % 64 == 0
//   * tcgen05 GEMM (gemm_tcgen05.cu) larger M, same dtype/shape conditions
//   * exact SIMT kernel (simt_linear.cu) fp32 activations and other shapes
// The LoRA down-projection runs first (lora_kernels.cu) into the workspace.
//
// Workspace layout (all offsets 256-byte aligned):
//   [0, 256)           arrival counters of split reductions (zero at rest)
//   [256, +M*r*4)      t = x.A^T (forward) or gt = (dy*s).B (dx)
//   [.., +P*4)         fp32 partials of the split LoRA reduction
#include <cuda_runtime.h>

#include "rq_internal.h"

namespace rq {

bool gemm_supported(const LinearArgs& a, bool dx);
int gemm_forward(const LinearArgs& a, const void* tdown, cudaStream_t st);
int gemm_dx(const LinearArgs& a, const void* gt, cudaStream_t st);
int lora_down_tc(int dt, bool wt, const void* X, int64_t M, int64_t Kr, const void* W2, int R, float pre_s,
                 bool do_pre, void* out, cudaStream_t st);

// The LoRA down product: on the tensor cores for prefill-sized M where it
// applies (gemm_tcgen05.cu), else the mma.sync / CUDA-core kernels.
static int lora_down_any(const LinearArgs& a, bool wt, const void* X, int64_t Kr, const void* W2, float pre_s,
                         bool do_pre, const struct WsView& v, cudaStream_t st);

static int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

static thread_local int t_last_path = RQ_PATH_NONE;
int last_path() { return t_last_path; }
constexpr int64_t kLoraSplitMax = 128;

int64_t linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int r) {
  (void)N;
  (void)K;
  if (r <= 0) return 256;
  const int64_t t_bytes = align256(M * r * 4);
  const int64_t m_small = M < 16 ? M : 16;
  const int64_t p_bytes = align256(kLoraSplitMax * m_small * r * 4);
  return 256 + t_bytes + p_bytes;
}

struct WsView {
  unsigned* counters;
  void* t;
  float* partial;
  int64_t partial_elems;
};

static int lora_down_any(const LinearArgs& a, bool wt, const void* X, int64_t Kr, const void* W2, float pre_s,
                         bool do_pre, const WsView& v, cudaStream_t st) {
  const int rc = lora_down_tc(a.xdt, wt, X, a.M, Kr, W2, a.r, pre_s, do_pre, v.t, st);
  if (rc != RQ_ERR_UNSUPPORTED) return rc;
  return lora_down(a.xdt, wt, X, a.M, Kr, W2, a.r, pre_s, do_pre, v.t, v.partial, v.partial_elems, v.counters, 64,
                   st);
}

static int carve(const LinearArgs& a, WsView* v) {
  v->counters = nullptr;
  v->t = nullptr;
  v->partial = nullptr;
  v->partial_elems = 0;
  if (a.r <= 0) return RQ_OK;
  const int64_t need = linear_workspace_bytes(a.M, a.w.N, a.w.K, a.r);
  if (a.ws == nullptr || a.ws_bytes < need) return RQ_ERR_WORKSPACE;
  if ((uintptr_t)a.ws % 256) return RQ_ERR_ALIGN;
  char* base = static_cast<char*>(a.ws);
  v->counters = reinterpret_cast<unsigned*>(base);
  v->t = base + 256;
  v->partial = reinterpret_cast<float*>(base + 256 + align256(a.M * a.r * 4));
  v->partial_elems = (a.ws_bytes - 256 - align256(a.M * a.r * 4)) / 4;
  return RQ_OK;
}

// Runs the GEMV over M in slabs of 16 rows (x, y and t advance together).
static int gemv_slabs(const LinearArgs& a, const void* t, cudaStream_t st) {
  const int es = a.xdt == RQ_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < a.M; m0 += 16) {
    LinearArgs s = a;
    s.M = a.M - m0 < 16 ? a.M - m0 : 16;
    s.x = static_cast<const char*>(a.x) + m0 * a.w.K * es;
    s.y = static_cast<char*>(a.y) + m0 * a.w.N * es;
    const void* ts = t ? static_cast<const char*>(t) + m0 * a.r * es : nullptr;
    const int rc = gemv_forward(s, ts, st);
    if (rc != RQ_OK) return rc;
  }
  return RQ_OK;
}

// The fused gather exists for the NF4 decode GEMV only; decided before any
// launch so that a caller can fall back to a collective.
static bool gather_eligible(const LinearArgs& a) {
  if (!is_nf4_fmt(a.w.fmt) || a.M < 1 || a.M > 16 || !gemv_supported(a)) return false;
  const RqGather& g = *a.gather;
  if (g.world < 1 || g.world > 64 || g.rank < 0 || g.rank >= g.world || !g.outs || !g.flags || !g.my_flags || !g.ctrl)
    return false;
  return g.col >= 0 && g.ld >= g.col + a.w.N;
}

int linear_forward(const LinearArgs& a, cudaStream_t st) {
  WsView v;
  t_last_path = RQ_PATH_NONE;
  if (a.gather && !gather_eligible(a)) return RQ_ERR_UNSUPPORTED;
  int rc = carve(a, &v);
  if (rc != RQ_OK) return rc;
  if (a.M == 0 || a.w.N == 0) return RQ_OK;
  LinearArgs g = a;
  g.M = a.M < 16 ? a.M : 16;
  const bool gemv = gemv_supported(g);
  if (gemv && a.M <= 16 && gemv_fuse_down(a)) {
    // one launch: the NF4 GEMV's grid computes x.A^T beside the main loop
    t_last_path = RQ_PATH_GEMV;
    return gemv_forward(a, v.t, st, v.partial, v.counters);
  }
  if (a.r > 0) {
    rc = lora_down_any(a, false, a.lora_x, a.w.K, a.lora_a, 1.0f, false, v, st);
    if (rc != RQ_OK) return rc;
  }
  if (gemv) {
    if (a.M <= 16) {
      t_last_path = RQ_PATH_GEMV;
      return gemv_forward(a, v.t, st);
    }
    if (gemm_supported(a, false)) {
      t_last_path = RQ_PATH_GEMM;
      return gemm_forward(a, v.t, st);
    }
    t_last_path = RQ_PATH_GEMV_SLABS;
    return gemv_slabs(a, v.t, st);
  }
  t_last_path = RQ_PATH_SIMT;
  return simt_forward(a, v.t, st);
}

int linear_dx(const LinearArgs& a, cudaStream_t st) {
  WsView v;
  t_last_path = RQ_PATH_NONE;
  int rc = carve(a, &v);
  if (rc != RQ_OK) return rc;
  if (a.M == 0 || a.w.K == 0) return RQ_OK;
  if (a.r > 0) {
    // gt = rnd(rnd(dy * s) . B): B is [N, r], the reduction runs over N
    rc = lora_down_any(a, true, a.x, a.w.N, a.lora_b, a.scaling, true, v, st);
    if (rc != RQ_OK) return rc;
  }
  if (gemm_supported(a, true)) {
    t_last_path = RQ_PATH_GEMM;
    return gemm_dx(a, v.t, st);
  }
  t_last_path = RQ_PATH_SIMT;
  return simt_dx(a, v.t, st);
}

}  // namespace rq
