"""FP8 compute over quantized storage (the reference's
rocm_qlora/fp8/fp8_linear.py: _FP8LinearFunc, FP8LinearWrapper,
wrap_model_for_fp8, enable_fp8_autocast; same names and results).

Storage stays QuantLinear (NF4 / INT8, double-quantized or not); the base
product runs as a per-tensor scaled FP8 GEMM, the adapter in the activation
dtype.  The native path computes what the reference's does
(fp8_linear.py:27-39, 98-114):

    w      = deq(W).to(x.dtype)
    w_s    = max|w| / 448          x_s = max|x| / 448          (fp32)
    y      = _scaled_mm(e4m3(x / x_s), e4m3(w / w_s).T, x_s, w_s) + bias
    out    = y + ((dropout(x) @ A.T) @ B.T) * scaling

with these differences in how, not what:
  * e4m3(w / w_s) and max|w| come from two passes over the codes on the GPU
    (rq_weight_absmax, rq_weight_to_fp8): no fp32 or bf16 copy of the weight
    is made, and the result is kept until the quantized buffers change (the
    base weight of a QLoRA layer is frozen; the reference re-dequantizes it
    on every call).  The division rounds as torch's GPU division of a bf16 /
    f16 tensor by a 0-dim fp32 tensor does: w_s converted to the tensor's
    dtype first;
  * x_s stays on the device (the reference's .item() syncs the host);
  * the backward's grad_x = grad_y @ w is the library's dX kernel over the
    codes (rq_linear_dx), not a matmul with a materialized weight;
  * the NaN check after _scaled_mm is gone: it caught the fnuz FP8 GEMM of
    ROCm returning NaN, which e4m3fn on NVIDIA tensor cores does not do.
Shapes _scaled_mm does not take (in / out features not multiples of 16) and
inputs off the GPU run the wrapped layer unchanged.
"""
import contextlib
import os
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn as nn

from rocm_qlora import _native as nat
from rocm_qlora.fp8.fp8_config import FP8Config, detect_fp8_support, get_fp8_dtype, get_fp8_recipe
from rocm_qlora.lora.lora_layer import LoRALinear
from rocm_qlora.quantization import layer_ops
from rocm_qlora.quantization.quant_linear import QuantLinear

_FP8_MAX = 448.0  # largest float8_e4m3fn value
_fp8_max_t: Dict[torch.device, torch.Tensor] = {}


def _fp8_max_on(dev: torch.device) -> torch.Tensor:
    """448 as a 0-dim fp32 tensor on dev: dividing by it is an IEEE fp32
    division (dividing by the Python number takes torch's scalar path, a
    multiplication by the reciprocal, which can be one ulp off)."""
    t = _fp8_max_t.get(dev)
    if t is None:
        t = _fp8_max_t[dev] = torch.full((), _FP8_MAX, dtype=torch.float32, device=dev)
    return t


def weight_fp8(w: layer_ops.WeightView, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """(e4m3fn [N, K], fp32 scale) of the quantized weight rounded to dtype:
    scale = max|w| / 448, codes e4m3fn(rnd(w / scale))."""
    L = nat.lib()
    dev = w.device
    with torch.cuda.device(dev):
        st = nat.stream_ptr(dev)
        amax = torch.empty(1, dtype=torch.float32, device=dev)
        nat.check(L.rq_weight_absmax(*w.args(), nat.dtype_code(dtype), amax.data_ptr(), st), "rq_weight_absmax")
        # as the reference: the maximum as a Python float, divided in double,
        # stored as fp32 (the same value as the fp32 division: the maximum
        # has at most 24 significant bits and 448 = 7 * 64)
        scale = float(amax.item()) / _FP8_MAX
        w_scale = torch.tensor(scale, dtype=torch.float32, device=dev)
        out = torch.empty(w.N, w.K, dtype=torch.float8_e4m3fn, device=dev)
        nat.check(L.rq_weight_to_fp8(*w.args(), nat.dtype_code(dtype), float(w_scale.item()),
                                     out.data_ptr(), st), "rq_weight_to_fp8")
    return out, w_scale


class _FP8LinearFunc(torch.autograd.Function):
    """FP8 forward of the frozen base product, grad_x in the activation dtype
    (the base weight is frozen, so no grad_w)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: layer_ops.WeightView, w_f8: torch.Tensor, w_scale: torch.Tensor,
                bias: Optional[torch.Tensor]) -> torch.Tensor:
        ctx.w = w
        ctx.x_shape = x.shape
        x2 = x.reshape(-1, x.shape[-1])
        f8 = get_fp8_dtype("e4m3")
        # max|x| / 448 correctly rounded to fp32, as the reference's
        # double division of .item() stored as fp32 (no host sync here)
        x_scale = (x2.abs().amax().float() / _fp8_max_on(x.device)).reshape(())
        x_f8 = (x2 / x_scale).to(f8)
        out = torch._scaled_mm(x_f8, w_f8.t(), scale_a=x_scale, scale_b=w_scale, out_dtype=x.dtype)
        out = out.reshape(*x.shape[:-1], -1)
        if bias is not None:
            out = out + bias
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        w = ctx.w
        gx = None
        if ctx.needs_input_grad[0]:
            gx = layer_ops.dx(w, grad_output.reshape(-1, w.N).contiguous(), None, None, 1.0).view(ctx.x_shape)
        return gx, None, None, None, None


class FP8LinearWrapper(nn.Module):
    """Wraps a LoRALinear to run its base product in FP8 while keeping the
    quantized storage; the adapter stays in the activation dtype."""

    def __init__(self, base_lora_linear: nn.Module, config: Optional[FP8Config] = None):
        super().__init__()
        self.config = config if config is not None else FP8Config()
        self.base = base_lora_linear
        self.fp8_info = detect_fp8_support()
        if not self.config.enabled or not self.fp8_info["fp8_supported"]:
            self.backend = "bf16"
        elif self.fp8_info["transformer_engine_available"] and self.config.use_transformer_engine:
            self.backend = "transformer_engine"
            self.te_recipe = get_fp8_recipe(self.config)
        elif self.fp8_info["fp8_dtypes_available"]:
            self.backend = "native"
        else:
            self.backend = "bf16"
        self._cache = None  # (WeightView, dtype, e4m3 weight, scale)

    def _fp8_operand(self, ql: QuantLinear, dtype: torch.dtype):
        w = ql.weight_view()
        c = self._cache
        if c is None or c[0] is not w or c[1] != dtype:
            w_f8, w_scale = weight_fp8(w, dtype)
            c = self._cache = (w, dtype, w_f8, w_scale)
        return c

    def _native_ok(self, x: torch.Tensor) -> bool:
        ql = getattr(self.base, "base_layer", None)
        return (isinstance(ql, QuantLinear) and x.is_cuda and ql.weight_quant.is_cuda and
                x.dtype in (torch.bfloat16, torch.float16) and not ql.merged_mode and
                not getattr(self.base, "merged", False) and
                ql.in_features % 16 == 0 and ql.out_features % 16 == 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.backend == "transformer_engine":
            import transformer_engine.pytorch as te
            with te.fp8_autocast(enabled=True, fp8_recipe=self.te_recipe):
                return self.base(x)
        if self.backend == "native" and self._native_ok(x):
            ql = self.base.base_layer
            w, _, w_f8, w_scale = self._fp8_operand(ql, x.dtype)
            bias = ql.bias.to(x.dtype) if ql.bias is not None else None
            base_out = _FP8LinearFunc.apply(x, w, w_f8, w_scale, bias)
            b = self.base
            lora_out = b.lora_dropout(x) @ b.lora_A.t().to(x.dtype) @ b.lora_B.t().to(x.dtype) * b.scaling
            return base_out + lora_out.to(base_out.dtype)
        return self.base(x)

    def extra_repr(self) -> str:
        return f"backend={self.backend}, fp8_supported={self.fp8_info['fp8_supported']}"


def wrap_model_for_fp8(model: nn.Module, config: Optional[FP8Config] = None) -> Tuple[nn.Module, Dict[str, Any]]:
    """Wraps every LoRALinear of the model in an FP8LinearWrapper; returns
    (model, {"enabled", "backend", "layers_wrapped", "reason"})."""
    config = config if config is not None else FP8Config()
    fp8_info = detect_fp8_support()
    status = {"enabled": False, "backend": "bf16", "layers_wrapped": 0, "reason": fp8_info["reason"]}
    if not fp8_info["fp8_supported"] and config.enabled:
        return model, status
    to_replace = [(name, m) for name, m in model.named_modules() if isinstance(m, LoRALinear)]
    for name, module in to_replace:
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        wrapped = FP8LinearWrapper(module, config)
        setattr(parent, child, wrapped)
        status["layers_wrapped"] += 1
        status["backend"] = wrapped.backend
        status["enabled"] = wrapped.backend != "bf16"
    if status["enabled"]:
        # the reference also raises the NCCL stream priority here (its other
        # setting, GPU_MAX_HW_QUEUES, is an AMD runtime variable)
        os.environ.setdefault("TORCH_NCCL_HIGH_PRIORITY", "1")
    return model, status


def enable_fp8_autocast(model: nn.Module, config: Optional[FP8Config] = None):
    """TransformerEngine's fp8_autocast when TE is installed and chosen, else
    a context that does nothing."""
    config = config if config is not None else FP8Config()
    try:
        import transformer_engine.pytorch as te
        if config.use_transformer_engine:
            return te.fp8_autocast(enabled=True, fp8_recipe=get_fp8_recipe(config))
    except Exception:
        pass
    return contextlib.nullcontext()
