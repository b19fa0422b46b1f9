/*
 * rq_b200.h -- C ABI of the B200 (sm_100a) implementation of rocm-qlora's
 * quantize / dequantize / QuantLinear+LoRA hot path.
 *
 * Conventions (every rq_* entry point):
 *   - plain device pointers and sizes; no framework types;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - nothing is allocated: callers own inputs, outputs and workspace;
 *   - the return value is RQ_OK (0) or a negative RQ_ERR_* status; the
 *     arguments are validated on the host before any launch, and a launch
 *     failure is reported as RQ_ERR_CUDA (rq_last_cuda_error() has the code);
 *   - calls are asynchronous on `stream` and thread-safe for distinct
 *     streams; a workspace must not be shared by calls that may overlap.
 *
 * Dtype codes: RQ_F32, RQ_BF16, RQ_F16.  Weight formats: RQ_W_* below.
 * Layouts follow the reference exactly (rocm_qlora/quantization):
 *   NF4 codes: flat row-major [N*K] elements, padded with zeros to a multiple
 *     of block_size, two codes per byte, byte i = code[2i] | code[2i+1] << 4;
 *   NF4 scales: one absmax per block, in the weight's dtype;
 *   double quant: c2 = one fp8-e4m3fnuz (or int8) byte per block, padded to a
 *     multiple of 256; c2_scales = fp32 absmax per 256 blocks;
 *   INT8 blockwise: int8 [N*K padded], scales per block (weight dtype);
 *   INT8 per-row: int8 [N, K], scales [N] (weight dtype).
 */
#ifndef RQ_B200_H
#define RQ_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define RQ_API __attribute__((visibility("default")))
#else
#define RQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RQ_OK 0
#define RQ_ERR_INVALID (-1)     /* bad size, null pointer, bad parameter */
#define RQ_ERR_ALIGN (-2)       /* pointer not aligned as required */
#define RQ_ERR_DTYPE (-3)       /* unsupported dtype / format code */
#define RQ_ERR_CUDA (-4)        /* CUDA launch or runtime error */
#define RQ_ERR_WORKSPACE (-5)   /* workspace missing or too small */
#define RQ_ERR_DEVICE (-6)      /* current device is not sm_100 */
#define RQ_ERR_SCRATCH (-7)     /* needs more than rq_linear_forward_noalloc's built-in scratch */
#define RQ_ERR_UNSUPPORTED (-8) /* no fused form for these arguments: nothing was launched */

#define RQ_F32 0
#define RQ_BF16 1
#define RQ_F16 2

#define RQ_W_NF4 0          /* NF4 codes + per-block scales */
#define RQ_W_NF4_DQ_FP8 1   /* NF4 codes + fp8-e4m3fnuz c2 + fp32 c2_scales */
#define RQ_W_NF4_DQ_INT8 2  /* NF4 codes + int8 c2 + fp32 c2_scales */
#define RQ_W_INT8 3         /* int8 blockwise */
#define RQ_W_INT8_ROW 4     /* int8 per output row (per_channel=True) */

/* ------------------------------------------------------------ utilities */
RQ_API int rq_abi_version(void);                 /* bumps on any ABI change */
RQ_API const char* rq_status_string(int status);
/* cudaError_t of the last RQ_ERR_CUDA in this thread, or 10000 + the CUresult
 * when a driver call (tensor-map encoding) failed */
RQ_API int rq_last_cuda_error(void);
/* Number of bounded in-kernel waits that ran out on the current device since
 * the last call (and reset it).  Nonzero means a kernel stopped early and its
 * output is not valid; it indicates a bug, never a normal condition.
 * Synchronous. */
RQ_API int rq_take_kernel_timeouts(unsigned int* count);

/* -------------------------------------------------------- quantization */

/* NF4 blockwise quantization of x[numel] (dtype RQ_F32/BF16/F16).
 * packed: ceil(numel/bs)*bs/2 bytes; scales: ceil(numel/bs) values of dtype.
 * block_size must be even and >= 2.
 * Replaces quantize_int4, rocm_qlora/quantization/quant_ops.py:80-126. */
RQ_API int rq_nf4_quantize(const void* x, int dtype, int64_t numel, int block_size,
                    uint8_t* packed, void* scales, void* stream);

/* NF4 dequantization of `nbytes` packed bytes (2*nbytes values) with
 * per-block scales of scale_dtype into out (out_dtype; RQ_F32 gives the
 * reference's fp32 result, RQ_BF16/RQ_F16 that value rounded).
 * Replaces dequantize_int4, quant_ops.py:128-150, and
 * dequantize_nf4_triton, rocm_qlora/kernels/nf4_dequant.py:81-115. */
RQ_API int rq_nf4_dequantize(const uint8_t* packed, int64_t nbytes, const void* scales,
                      int scale_dtype, int block_size, void* out, int out_dtype,
                      void* stream);

/* INT8 blockwise quantization: q[ceil(numel/bs)*bs], scales[ceil(numel/bs)].
 * Replaces quantize_int8(per_channel=False), quant_ops.py:36-53. */
RQ_API int rq_int8_quantize(const void* x, int dtype, int64_t numel, int block_size,
                     int8_t* q, void* scales, void* stream);

/* INT8 per-row quantization of x[rows, cols]: q[rows, cols], scales[rows].
 * Replaces quantize_int8(per_channel=True), quant_ops.py:28-35. */
RQ_API int rq_int8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t cols,
                          int8_t* q, void* scales, void* stream);

/* INT8 dequantization of q[numel]; cols > 0 selects per-row scales (row =
 * i / cols), else blockwise with block_size.
 * Replaces dequantize_int8, quant_ops.py:55-78. */
RQ_API int rq_int8_dequantize(const int8_t* q, int64_t numel, const void* scales,
                       int scale_dtype, int block_size, int64_t cols, void* out,
                       int out_dtype, void* stream);

/* Second-level quantization of nb fp32 first-level scales c1:
 * c2[ceil(nb/block2)*block2] (fp8 e4m3fnuz bytes if fp8 != 0, else int8),
 * c2_scales[ceil(nb/block2)] fp32.
 * Replaces double_quantize lines 58-97, rocm_qlora/quantization/double_quant.py. */
RQ_API int rq_dq_quantize_scales(const float* c1, int64_t nb, int block2, int fp8,
                          uint8_t* c2, float* c2_scales, void* stream);

/* Double-quantized NF4 dequantization of `numel` values:
 * out[i] = T[code_i] * (c2[i/bs] * c2_scales[i/bs/block2]).
 * Replaces double_dequantize, double_quant.py:99-122. */
RQ_API int rq_dq_dequantize(const uint8_t* packed, int64_t numel, const uint8_t* c2,
                     const float* c2_scales, int fp8, int block_size, int block2,
                     void* out, int out_dtype, void* stream);

/* ------------------------------------------------ QuantLinear + LoRA */

/* Bytes of workspace rq_linear_forward / rq_linear_dx need for these sizes
 * (0 is possible).  The first 256 bytes of a workspace are a counter area
 * that must be zero before its first use; the kernels leave it zero. */
RQ_API int64_t rq_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int r);

/* y[M,N] = base + lora where, in the activation dtype `xdtype`,
 *   base = round(x[M,K] . deq(W)^T + bias)          (fp32 accumulation)
 *   lora = round(round(round(x . A^T) . B^T) * scaling)
 *   y    = round(base + lora)
 * i.e. LoRALinear.forward in eval mode over QuantLinear.forward
 * (rocm_qlora/lora/lora_layer.py:51-70, quantization/quant_linear.py:121-197,
 * kernels/dequant_matmul.py:356-376).  W is [N, K] in format `wfmt`:
 *   qweight  NF4 packed codes / int8 values (layout above);
 *   scales   per-block (or per-row) scales of scale_dtype (unused for DQ);
 *   c2, c2_scales  double-quant second level (DQ formats only).
 * bias [N] (bias_dtype) may be NULL; lora_a [r,K] and lora_b [N,r] are in
 * xdtype and may both be NULL (r = 0).  lora_x [M,K] is the input of the
 * adapter branch when it differs from x (LoRA dropout in training,
 * lora_layer.py:67); NULL means x.  x, y contiguous row-major.
 * xdtype: RQ_BF16 or RQ_F16 (tensor-core paths) or RQ_F32. */
RQ_API int rq_linear_forward(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                      const uint8_t* c2, const float* c2_scales,
                      int64_t N, int64_t K, int block_size,
                      const void* x, int xdtype, int64_t M, const void* lora_x,
                      const void* bias, int bias_dtype,
                      const void* lora_a, const void* lora_b, int r, float scaling,
                      void* y, void* workspace, int64_t workspace_bytes, void* stream);

/* dx[M,K] = round(round(dy . deq(W)) + round(round(round(dy*scaling) . B) . A)),
 * the input gradient of the same layer (autograd of lora_layer.py:67 with a
 * frozen base; kernels/dequant_matmul.py:337-351 for the base term). */
RQ_API int rq_linear_dx(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                 const uint8_t* c2, const float* c2_scales,
                 int64_t N, int64_t K, int block_size,
                 const void* dy, int xdtype, int64_t M,
                 const void* lora_a, const void* lora_b, int r, float scaling,
                 void* dx, void* workspace, int64_t workspace_bytes, void* stream);

/* The merged weight of a LoRA-adapted layer, dequantized and combined with
 * the adapter in one pass over the codes:
 *   out[n, k] = deq(W)[n, k] + scaling * sum_j lora_b[n, j] * lora_a[j, k]
 * with lora_a [r, K] and lora_b [N, r] fp32 (the adapters' parameter dtype)
 * and out [N, K] row-major in out_dtype.  mode RQ_MERGE_FP32_SUM adds in
 * fp32 and rounds once (LoRALinear.merge_lora, rocm_qlora/lora/
 * lora_layer.py:72-113); RQ_MERGE_ROUND_EACH rounds the weight and the delta
 * to out_dtype first and adds them there (_export_dequant_layer,
 * rocm_qlora/export/gguf_export.py:30-80).  r = 0 gives the dequantized
 * weight alone (lora_a / lora_b may then be NULL).  r <= 128. */
#define RQ_MERGE_FP32_SUM 0
#define RQ_MERGE_ROUND_EACH 1
RQ_API int rq_merge_lora(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                  const uint8_t* c2, const float* c2_scales,
                  int64_t N, int64_t K, int block_size,
                  const float* lora_a, const float* lora_b, int r, float scaling, int mode,
                  void* out, int out_dtype, void* stream);

/* The quantized weight as a per-tensor scaled float8_e4m3fn GEMM operand
 * (FP8LinearWrapper's native path, rocm_qlora/fp8/fp8_linear.py:27-39):
 *   rq_weight_absmax: *absmax (device fp32) = max |rnd(deq(W))|, the weight
 *     rounded to `dtype` (the activation dtype, RQ_BF16 / RQ_F16 / RQ_F32);
 *   rq_weight_to_fp8: fp8_out[n*K + k] = e4m3fn(rnd(rnd(deq(W)[n, k]) / rnd(w_scale)))
 *     (as torch divides a `dtype` tensor by a 0-dim fp32 GPU tensor: the
 *     divisor rounded to `dtype`, the division in fp32 rounded to `dtype`;
 *     then round-to-nearest-even to e4m3fn without saturation), N*K bytes
 *     row-major.
 * The reference computes w_scale = absmax / 448 (e4m3fn's largest value). */
RQ_API int rq_weight_absmax(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                     const uint8_t* c2, const float* c2_scales,
                     int64_t N, int64_t K, int block_size, int dtype,
                     float* absmax, void* stream);
RQ_API int rq_weight_to_fp8(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                     const uint8_t* c2, const float* c2_scales,
                     int64_t N, int64_t K, int block_size, int dtype, float w_scale,
                     uint8_t* fp8_out, void* stream);

/* Bytes of device scratch compiled into the library for
 * rq_linear_forward_noalloc (held on every GPU that loads the library). */
#define RQ_NOALLOC_SCRATCH_BYTES (2u << 20)

/* rq_linear_forward for callers that cannot allocate device memory (plugin
 * hosts that own all device memory and hand out no workspace, cgo / JNI /
 * FFI bindings without a CUDA allocator, loops where cudaMalloc would
 * synchronize the device).  Same arguments and result as rq_linear_forward
 * minus the workspace: the scratch is a fixed RQ_NOALLOC_SCRATCH_BYTES
 * device array inside the library, so nothing is allocated.  Calls whose
 * rq_linear_workspace_bytes(M, N, K, r) exceeds that size return
 * RQ_ERR_SCRATCH before touching the GPU.  The first call on a device looks
 * up the array's device address (make it before any stream capture); after
 * cudaDeviceReset the next call looks it up again.  All
 * calls share the array: calls that may overlap on the GPU race and must not
 * be issued.  This entry point has no counterpart in the reference. */
RQ_API int rq_linear_forward_noalloc(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                      const uint8_t* c2, const float* c2_scales,
                      int64_t N, int64_t K, int block_size,
                      const void* x, int xdtype, int64_t M, const void* lora_x,
                      const void* bias, int bias_dtype,
                      const void* lora_a, const void* lora_b, int r, float scaling,
                      void* y, void* stream);

/* Numerics of the decode GEMV (M <= 16, NF4 formats).  0 (the default): the
 * NF4 levels enter the tensor-core multiply rounded once to the activation
 * dtype and the fp32 block scale multiplies each 64-wide partial sum.  The
 * reference instead rounds level x scale to the activation dtype per weight;
 * the two differ by a fixed error per code, within 1e-2 x RMS of the output
 * for centred activations, but adding up over K when the activations share
 * a sign (after a ReLU, say).  1 (exact): the kernel forms the reference's
 * own weights, fp32 level x fp32 scale rounded to the activation dtype, per
 * weight, so only the summation order differs; slower.  The environment
 * variable RQ_DECODE_EXACT=1 selects 1 at the first call.  Applies to
 * launches made after the call; no counterpart in the reference. */
RQ_API void rq_set_decode_exact(int exact);

/* Kernel family the last rq_linear_forward / rq_linear_dx of this thread
 * ran: RQ_PATH_GEMV (decode, M <= 16), RQ_PATH_GEMM (tcgen05 prefill GEMM),
 * RQ_PATH_GEMV_SLABS (the GEMV over 16-row slabs), RQ_PATH_SIMT (exact
 * CUDA-core kernel), RQ_PATH_NONE (nothing launched).  Introspection for
 * tests and tuning; no counterpart in the reference. */
#define RQ_PATH_NONE 0
#define RQ_PATH_GEMV 1
#define RQ_PATH_GEMM 2
#define RQ_PATH_GEMV_SLABS 3
#define RQ_PATH_SIMT 4
RQ_API int rq_last_path(void);

/* ------------------------------- column shards: fused output gather */

/* Device memory shared with the other ranks of one node (one process per
 * GPU, NVLink peers).  rq_peer_alloc returns a zero-filled cudaMalloc
 * allocation of `bytes` on the current device; rq_peer_handle writes its
 * 64-byte IPC handle to `handle` (the caller ships it to the other ranks);
 * rq_peer_open maps another rank's allocation into this process for the
 * current device (peer access enabled) and rq_peer_close unmaps it.
 * Plumbing for rq_linear_forward_gather; no counterpart in the reference,
 * which replicates layers instead of sharding them. */
RQ_API int rq_peer_alloc(int64_t bytes, void** ptr);
RQ_API int rq_peer_free(void* ptr);
RQ_API int rq_peer_handle(const void* ptr, void* handle);
RQ_API int rq_peer_open(const void* handle, void** ptr);
RQ_API int rq_peer_close(void* ptr);

/* The node-wide output of a column-sharded layer: every rank computes the
 * output features [col, col + N) of the full Y[M, ld] and writes them into
 * EVERY rank's copy of Y.  All pointers are device pointers valid on this
 * rank (peer allocations opened with rq_peer_open):
 *   outs[q]      rank q's Y (row stride ld elements of xdtype), q < world
 *   flags[q]     rank q's flag array, 2 * world uint32 (zero before first
 *                use): [0, world) the epoch each rank finished, [world,
 *                2 * world) the epoch each rank entered
 *   my_flags     this rank's flag array (== flags[rank])
 *   ctrl         this rank's 4 uint32 of control state, zero before first
 *                use: [0] arrival counter (kernels leave it zero), [1] epoch
 *                (calls so far), [2] error (set to 1 if a peer did not
 *                arrive within about 2 s; the output is then incomplete)
 * outs and flags are device arrays of `world` pointers. */
typedef struct RqGather {
  void* const* outs;
  uint32_t* const* flags;
  uint32_t* my_flags;
  uint32_t* ctrl;
  int64_t ld;
  int64_t col;
  int world;
  int rank;
} RqGather;

/* rq_linear_forward of this rank's shard (W is [N, K], the shard's rows)
 * whose output is written into every rank's Y[:, col:col+N] instead of a
 * local y; when the kernel has completed on a rank, every rank's shard of
 * this call is in that rank's Y (the ranks meet at the end of the kernel:
 * the last CTA publishes this call's epoch to every rank's flags and waits,
 * bounded, for all of theirs).  Every rank must make the same sequence of
 * calls with the same M.  A rank's Y is rewritten by the next call that
 * names it, so each rank consumes each result (in stream order) before it
 * issues its next call on the same outputs; a rank writes into the other
 * ranks' Y only after every rank has entered the call (each rank announces
 * its entry at the start of the kernel), so a faster rank never overwrites
 * a result a slower rank is still reading.  Only the fused decode GEMV (NF4 formats, bf16/f16,
 * M <= 16) has this form: other arguments return RQ_ERR_UNSUPPORTED before
 * anything is launched, and the caller gathers with a collective instead.
 * Same-node NVLink peers only; one call in flight per RqGather. */
RQ_API int rq_linear_forward_gather(int wfmt, const void* qweight, const void* scales, int scale_dtype,
                      const uint8_t* c2, const float* c2_scales,
                      int64_t N, int64_t K, int block_size,
                      const void* x, int xdtype, int64_t M,
                      const void* bias, int bias_dtype,
                      const void* lora_a, const void* lora_b, int r, float scaling,
                      const RqGather* gather, void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------- reference launcher drop-ins */

/* Same symbol names, argument order and types as the reference's HIP
 * launchers (rocm_qlora/hip_kernels/int4_matmul.hip:413-458, bound by
 * ctypes in rocm_qlora/hip_kernels/build_utils.py:237-262): x fp16 [M,K],
 * scales fp16 per 64-block as declared there, c fp16 [M,N], no bias.  They
 * return void like the originals; the status of the last call is available
 * from rq_last_status(). */
RQ_API void launch_int4_dequant_matmul(void* stream, void* x, void* w_packed, void* scales,
                                void* c, int M, int N, int K, int block_size);
RQ_API void launch_int8_dequant_matmul(void* stream, void* x, void* w_int8, void* scales,
                                void* c, int M, int N, int K, int block_size);
RQ_API int rq_last_status(void);

#ifdef __cplusplus
}
#endif

#endif /* RQ_B200_H */
