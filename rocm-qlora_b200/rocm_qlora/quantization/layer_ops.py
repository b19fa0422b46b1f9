"""Autograd wrappers around the fused QuantLinear(+LoRA) kernels.

``QuantLinear.forward`` and ``LoRALinear.forward`` call into here; each call
is one ``rq_linear_forward`` (and, in backward, one ``rq_linear_dx``) on the
current CUDA stream, through the torch extension's operators
(``torch.ops.rocm_qlora.linear_forward`` / ``linear_dx``, csrc/torch_ops.cpp)
or, where that extension is not built, through ctypes.  The adapter gradients dA / dB are plain cuBLAS matmuls
in the activation dtype with the same roundings as the reference's autograd
of ``x @ A.T @ B.T * scaling`` (rocm_qlora/lora/lora_layer.py:67).
"""
import ctypes
import weakref
from dataclasses import dataclass
from typing import Optional

import torch

from rocm_qlora import _native as nat


@dataclass
class WeightView:
    """The quantized operand of a QuantLinear, as the C ABI takes it."""
    fmt: int
    q: torch.Tensor
    scales: Optional[torch.Tensor]
    c2: Optional[torch.Tensor]
    c2_scales: Optional[torch.Tensor]
    N: int
    K: int
    block_size: int

    @property
    def device(self) -> torch.device:
        return self.q.device

    def args(self):
        a = self.__dict__.get("_args")
        if a is None:  # the view is immutable: its pointers never change
            sc = self.scales
            a = (self.fmt, self.q.data_ptr(), nat.ptr(sc), nat.dtype_code(sc.dtype) if sc is not None else 0,
                 nat.ptr(self.c2), nat.ptr(self.c2_scales), self.N, self.K, self.block_size)
            self.__dict__["_args"] = a
        return a


def weight_view(ql) -> WeightView:
    """WeightView of a QuantLinear module (formats of quant_linear.py)."""
    N, K = ql.out_features, ql.in_features
    if ql.bits == 4:
        if getattr(ql, "use_double_quant", False):
            if not hasattr(ql, "c2") or not hasattr(ql, "c2_scales"):
                raise RuntimeError(
                    "Double quantization attributes not initialized. "
                    "Call patch_quant_linear_for_double_quant() first.")
            fmt = nat.W_NF4_DQ_FP8 if getattr(ql, "use_fp8_c2", True) else nat.W_NF4_DQ_INT8
            c2 = ql.c2.reshape(-1).view(torch.uint8)
            c2s = ql.c2_scales.reshape(-1).to(torch.float32)
            return WeightView(fmt, ql.weight_quant.reshape(-1), None, c2.contiguous(), c2s.contiguous(), N, K,
                              ql.block_size)
        return WeightView(nat.W_NF4, ql.weight_quant.reshape(-1), ql.weight_scales.reshape(-1).contiguous(),
                          None, None, N, K, ql.block_size)
    if ql.bits == 8:
        wq = ql.weight_quant
        sc = ql.weight_scales.reshape(-1).contiguous()
        if wq.dim() == 2 and sc.numel() == wq.size(0):
            return WeightView(nat.W_INT8_ROW, wq.contiguous(), sc, None, None, N, K, ql.block_size)
        return WeightView(nat.W_INT8, wq.reshape(-1), sc, None, None, N, K, ql.block_size)
    raise ValueError(f"Unsupported bit depth: {ql.bits}")


def _check_device(w: WeightView, x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise nat.NativeUnavailable(
            "rocm_qlora (B200 build) computes on the GPU only: move the input and the model to a CUDA device")
    if w.q.device != x.device:
        raise RuntimeError(f"QuantLinear buffers are on {w.q.device} but the input is on {x.device}")


_ws_bytes = {}  # rq_linear_workspace_bytes by (M, N, K, r): a pure function of them


def _split_adapter(M: int, r: int, dtype: torch.dtype, for_dx: bool) -> bool:
    """Whether the adapter term runs beside the kernel instead of inside it.
    The tensor-core GEMM (forward M >= 64, dX every M) takes ranks <= 64
    that are multiples of 8; other ranks would send those calls to the exact
    CUDA-core kernel (slow at these sizes).  They run the kernel without
    the adapter and add the adapter term with cuBLAS matmuls in the
    activation dtype, rounding as the reference does."""
    if r == 0 or (r <= 64 and r % 8 == 0) or dtype not in (torch.bfloat16, torch.float16):
        return False
    return for_dx or M >= 64


def forward(w: WeightView, x2d: torch.Tensor, bias: Optional[torch.Tensor], A: Optional[torch.Tensor],
            B: Optional[torch.Tensor], scaling: float, lora_x: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[M, N] of LoRALinear.forward (eval) over QuantLinear.forward."""
    L = nat.lib()
    _check_device(w, x2d)
    dev = x2d.device
    M = x2d.shape[0]
    dt = nat.dtype_code(x2d.dtype)
    r = 0 if A is None else A.shape[0]
    if _split_adapter(M, r, x2d.dtype, False):
        # rnd(base + rnd(rnd(rnd(x_l . A^T) . B^T) * s)), base = rnd(x . W^T (+ bias))
        base = forward(w, x2d, bias, None, None, 1.0)
        xin = lora_x if lora_x is not None else x2d
        return base + (xin @ A.t()) @ B.t() * scaling
    key = (M, w.N, w.K, r)
    nbytes = _ws_bytes.get(key)
    if nbytes is None:
        nbytes = _ws_bytes[key] = L.rq_linear_workspace_bytes(M, w.N, w.K, r)

    if nat.ops():
        # one dispatcher call: device guard, output, x's device's current
        # stream and the status check are in the extension
        return torch.ops.rocm_qlora.linear_forward(
            x2d, w.fmt, w.q, w.scales, w.c2, w.c2_scales, w.N, w.K, w.block_size, lora_x, bias, A, B,
            float(scaling), nat.workspace(dev, nbytes))
    y = torch.empty(M, w.N, dtype=x2d.dtype, device=dev)

    def call():
        st = nat.stream_ptr(dev)
        ws = nat.workspace(dev, nbytes, st)
        return L.rq_linear_forward(*w.args(), x2d.data_ptr(), dt, M, nat.ptr(lora_x), nat.ptr(bias),
                                   nat.dtype_code(bias.dtype) if bias is not None else 0, nat.ptr(A), nat.ptr(B),
                                   r, float(scaling), y.data_ptr(), ws.data_ptr(), ws.numel(), st)

    # the library launches on the current stream of x's device, which must
    # be the current device
    if dev.index == torch.cuda.current_device():
        rc = call()
    else:
        with torch.cuda.device(dev):
            rc = call()
    nat.check(rc, "rq_linear_forward")
    return y


# Adapter parameters cast to the activation dtype, kept between calls: the
# fp32 parameters would otherwise be cast (two kernels and two allocations)
# on every layer call.  An entry is valid while the parameter keeps its
# storage and in-place version (optimizer steps, copy_ and load_state_dict
# bump the version); writes through ``.data`` do not, so code that writes
# adapters that way calls forget_casts() (LoRALinear.merge_lora does).
# Nothing is cached while a CUDA graph is being captured: a cast made there
# only gets its values when the graph replays.
_casts = {}  # id(parameter) -> (weakref to it, version, data_ptr, dtype, cast)


def cast_param(p: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    """`p` in dtype `dt`, contiguous, reusing the last cast while valid."""
    if p.dtype == dt and p.is_contiguous():
        return p
    if p.is_cuda and torch.cuda.is_current_stream_capturing():
        return p.detach().to(dt).contiguous()
    key, ver, ptr = id(p), p._version, p.data_ptr()
    e = _casts.get(key)
    if e is not None and e[0]() is p and e[1] == ver and e[2] == ptr and e[3] == dt:
        return e[4]
    c = p.detach().to(dt).contiguous()
    _casts[key] = (weakref.ref(p, lambda _r, k=key: _casts.pop(k, None)), ver, ptr, dt, c)
    return c


def forget_casts(*params: torch.Tensor) -> None:
    """Drop the cached casts of `params` (after writes through ``.data``)."""
    for p in params:
        e = _casts.get(id(p))
        if e is not None and e[0]() is p:
            del _casts[id(p)]


def _lora_operands(x, lora_A, lora_B, xd, bias):
    """x and the adapter input as [M, K], A / B / bias in x's dtype."""
    K = x.shape[-1]
    dt = x.dtype
    x2 = x.reshape(-1, K).contiguous()
    xd2 = xd.reshape(-1, K).contiguous() if xd is not None else None
    A = cast_param(lora_A, dt)
    B = cast_param(lora_B, dt)
    b = bias.to(dt).contiguous() if bias is not None else None
    return x2, xd2, A, B, b


def lora_forward(x, lora_A, lora_B, xd, w: WeightView, bias, scaling) -> torch.Tensor:
    """LoRAQuantFunction's forward without autograd (nothing needs a
    gradient): the same kernel call, none of the Function bookkeeping."""
    x2, xd2, A, B, b = _lora_operands(x, lora_A, lora_B, xd, bias)
    return forward(w, x2, b, A, B, scaling, lora_x=xd2).view(*x.shape[:-1], w.N)


def quant_forward(x, w: WeightView, bias) -> torch.Tensor:
    """QuantLinearFunction's forward without autograd."""
    K = x.shape[-1]
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    return forward(w, x.reshape(-1, K).contiguous(), b, None, None, 1.0).view(*x.shape[:-1], w.N)


def forward_gather(w: WeightView, x2d: torch.Tensor, bias: Optional[torch.Tensor], A: Optional[torch.Tensor],
                   B: Optional[torch.Tensor], scaling: float, gather) -> int:
    """This rank's shard of a column-sharded layer written into every rank's
    output (``gather``: an ``_native.RqGather``).  Returns the library status:
    RQ_OK, or RQ_ERR_UNSUPPORTED when these arguments have no fused form
    (nothing was launched; the caller gathers with a collective).  Other
    errors raise."""
    L = nat.lib()
    _check_device(w, x2d)
    dev = x2d.device
    M = x2d.shape[0]
    r = 0 if A is None else A.shape[0]
    with torch.cuda.device(dev):
        nbytes = L.rq_linear_workspace_bytes(M, w.N, w.K, r)
        ws = nat.workspace(dev, nbytes)
        rc = L.rq_linear_forward_gather(*w.args(), x2d.data_ptr(), nat.dtype_code(x2d.dtype), M, nat.ptr(bias),
                                        nat.dtype_code(bias.dtype) if bias is not None else 0, nat.ptr(A), nat.ptr(B),
                                        r, float(scaling), ctypes.byref(gather), ws.data_ptr(), ws.numel(),
                                        nat.stream_ptr(dev))
    if rc != nat.RQ_ERR_UNSUPPORTED:
        nat.check(rc, "rq_linear_forward_gather")
    return rc


def dx(w: WeightView, dy2d: torch.Tensor, A: Optional[torch.Tensor], B: Optional[torch.Tensor],
       scaling: float) -> torch.Tensor:
    """dx[M, K] = rnd(rnd(dy . W) + rnd(rnd(rnd(dy*s) . B) . A))."""
    L = nat.lib()
    _check_device(w, dy2d)
    dev = dy2d.device
    M = dy2d.shape[0]
    r = 0 if A is None else A.shape[0]
    if _split_adapter(M, r, dy2d.dtype, True):
        return dx(w, dy2d, None, None, 1.0) + ((dy2d * scaling) @ B) @ A
    with torch.cuda.device(dev):
        nbytes = L.rq_linear_workspace_bytes(M, w.N, w.K, r)
        ws = nat.workspace(dev, nbytes)
        if nat.ops():
            return torch.ops.rocm_qlora.linear_dx(dy2d, w.fmt, w.q, w.scales, w.c2, w.c2_scales, w.N, w.K,
                                                  w.block_size, A, B, float(scaling), ws)
        out = torch.empty(M, w.K, dtype=dy2d.dtype, device=dev)
        nat.check(L.rq_linear_dx(*w.args(), dy2d.data_ptr(), nat.dtype_code(dy2d.dtype), M, nat.ptr(A), nat.ptr(B),
                                 r, float(scaling), out.data_ptr(), ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
                  "rq_linear_dx")
    return out


class QuantLinearFunction(torch.autograd.Function):
    """F.linear(x, deq(W).to(x.dtype), bias) with a frozen quantized weight."""

    @staticmethod
    def forward(ctx, x, w: WeightView, bias):
        K = x.shape[-1]
        x2 = x.reshape(-1, K).contiguous()
        b = bias.to(x.dtype).contiguous() if bias is not None else None
        y = forward(w, x2, b, None, None, 1.0)
        ctx.w = w
        ctx.x_shape = x.shape
        return y.view(*x.shape[:-1], w.N)

    @staticmethod
    def backward(ctx, gy):
        w = ctx.w
        gx = None
        if ctx.needs_input_grad[0]:
            gx = dx(w, gy.reshape(-1, w.N).contiguous(), None, None, 1.0).view(ctx.x_shape)
        return gx, None, None


class LoRAQuantFunction(torch.autograd.Function):
    """LoRALinear.forward over a QuantLinear base in one fused kernel.

    Inputs: x [..., K]; lora_A [r, K] and lora_B [N, r] (parameters, any
    float dtype, used in x.dtype); xd = the adapter input when LoRA dropout
    is active (else None, meaning x).  With xd given, x's gradient carries
    only the base term and xd's gradient the adapter term, so autograd adds
    them after the dropout backward exactly as in the reference."""

    @staticmethod
    def forward(ctx, x, lora_A, lora_B, xd, w: WeightView, bias, scaling):
        x2, xd2, A, B, b = _lora_operands(x, lora_A, lora_B, xd, bias)
        y = forward(w, x2, b, A, B, scaling, lora_x=xd2)
        ctx.save_for_backward(x2 if xd2 is None else xd2, A, B)
        ctx.w, ctx.scaling, ctx.has_xd = w, scaling, xd is not None
        ctx.x_shape = x.shape
        ctx.param_dtypes = (lora_A.dtype, lora_B.dtype)
        return y.view(*x.shape[:-1], w.N)

    @staticmethod
    def backward(ctx, gy):
        xin, A, B = ctx.saved_tensors
        w, s = ctx.w, ctx.scaling
        dy = gy.reshape(-1, w.N).contiguous()
        gx = gA = gB = gxd = None
        need_x, need_A, need_B, need_xd = ctx.needs_input_grad[:4]
        if need_x:
            if ctx.has_xd:
                gx = dx(w, dy, None, None, 1.0).view(ctx.x_shape)
            else:
                gx = dx(w, dy, A, B, s).view(ctx.x_shape)
        if need_A or need_B or need_xd:
            gu = dy * s                      # grad of (u * scaling), rounded to dt
            gt = gu @ B                      # grad of t = x @ A.T      [M, r]
            if need_B:
                t = xin @ A.t()
                gB = (gu.t() @ t).to(ctx.param_dtypes[1])
            if need_A:
                gA = (gt.t() @ xin).to(ctx.param_dtypes[0])
            if need_xd and ctx.has_xd:
                gxd = (gt @ A).view(ctx.x_shape)
        return gx, gA, gB, gxd, None, None, None


MERGE_FP32_SUM, MERGE_ROUND_EACH = 0, 1


def merge_weight(w: WeightView, A: Optional[torch.Tensor], B: Optional[torch.Tensor], scaling: float, mode: int,
                 out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """[N, K] weight deq(W) + scaling * B @ A in one kernel pass (rq_merge_lora):
    mode MERGE_FP32_SUM adds in fp32 and rounds once (merge_lora),
    MERGE_ROUND_EACH rounds both terms to out_dtype before adding
    (_export_dequant_layer).  A [r, K] and B [N, r] are used as fp32."""
    L = nat.lib()
    dev = w.device
    r = 0 if A is None else A.shape[0]
    out = torch.empty(w.N, w.K, dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        A32 = A.detach().to(device=dev, dtype=torch.float32).contiguous() if r else None
        B32 = B.detach().to(device=dev, dtype=torch.float32).contiguous() if r else None
        nat.check(L.rq_merge_lora(*w.args(), nat.ptr(A32), nat.ptr(B32), r, float(scaling), mode, out.data_ptr(),
                                  nat.dtype_code(out_dtype), nat.stream_ptr(dev)), "rq_merge_lora")
    return out
