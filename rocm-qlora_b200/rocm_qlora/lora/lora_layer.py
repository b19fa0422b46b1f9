"""LoRALinear: trainable low-rank adapters around a QuantLinear.

Same API and initialisation as the reference (rocm_qlora/lora/lora_layer.py:
17-135).  Over a QuantLinear base the whole forward -- dequantize, matmul,
bias, ``x @ A.T @ B.T * scaling`` and the final add -- is one call into the
fused kernel, with the reference's rounding of each intermediate to the
activation dtype; the backward's input gradient is one call as well.
"""
import math

import torch
import torch.nn as nn

from rocm_qlora.quantization.quant_linear import QuantLinear
from rocm_qlora.quantization import layer_ops


class LoRALinear(nn.Module):
    """Wraps a QuantLinear with LoRA adapters A [r, in] and B [out, r]."""

    def __init__(self, quant_linear: QuantLinear, r: int = 8, lora_alpha: int = 16, lora_dropout: float = 0.0):
        super().__init__()
        self.base_layer = quant_linear
        self.r = r
        self.lora_alpha = lora_alpha
        self.merged = False
        for p in self.base_layer.parameters():
            p.requires_grad_(False)
        self.lora_A = nn.Parameter(torch.empty(r, quant_linear.in_features))
        self.lora_B = nn.Parameter(torch.zeros(quant_linear.out_features, r))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))  # PEFT convention; B = 0 -> no-op at init
        self.scaling = lora_alpha / r
        self.lora_dropout = nn.Dropout(p=lora_dropout) if lora_dropout > 0.0 else nn.Identity()

    def _fusable(self) -> bool:
        b = self.base_layer
        return isinstance(b, QuantLinear) and not (b.merged_mode and b.merged_fp16_weight is not None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """base_output + (dropout(x) @ A.T @ B.T * scaling)."""
        if self.merged:
            return self.base_layer(x)
        if self._fusable():
            xd = None
            if isinstance(self.lora_dropout, nn.Dropout) and self.training and self.lora_dropout.p > 0:
                xd = self.lora_dropout(x)
            b = self.base_layer
            if torch.is_grad_enabled() and (x.requires_grad or self.lora_A.requires_grad or
                                            self.lora_B.requires_grad or (xd is not None and xd.requires_grad)):
                return layer_ops.LoRAQuantFunction.apply(x, self.lora_A, self.lora_B, xd, b.weight_view(), b.bias,
                                                         self.scaling)
            return layer_ops.lora_forward(x, self.lora_A, self.lora_B, xd, b.weight_view(), b.bias, self.scaling)
        # any other base module: the reference's composition, unchanged
        if hasattr(self.base_layer, 'weight'):
            base_out = self.base_layer(x.to(self.base_layer.weight.dtype))
        else:
            base_out = self.base_layer(x)
        lora_out = self.lora_dropout(x) @ self.lora_A.to(x.dtype).T @ self.lora_B.to(x.dtype).T * self.scaling
        return base_out + lora_out.to(base_out.dtype)

    def merge_lora(self) -> None:
        """Store W + B @ A * scaling as an fp16 weight (no re-quantization)
        and zero the adapters; unmerge_lora() reverts.  On the GPU the merged
        weight comes from one kernel pass over the codes (rq_merge_lora)."""
        if self.merged:
            raise RuntimeError("LoRA already merged")
        b = self.base_layer
        if isinstance(b, QuantLinear) and b.weight_quant.is_cuda:
            # dequantize, B @ A * scaling and the fp32 add in one pass over the codes
            merged_weight = layer_ops.merge_weight(b.weight_view(), self.lora_A, self.lora_B, self.scaling,
                                                   layer_ops.MERGE_FP32_SUM, torch.float16)
        else:
            delta_W = (self.lora_B @ self.lora_A) * self.scaling
            base_weight_fp = b.dequantized_weight()
            merged_weight = (base_weight_fp + delta_W.to(base_weight_fp.dtype)).to(torch.float16)
        self.base_layer.merged_fp16_weight = merged_weight
        self.base_layer.merged_mode = True
        self.merged = True
        self.lora_A.data.zero_()
        self.lora_B.data.zero_()
        layer_ops.forget_casts(self.lora_A, self.lora_B)

    def unmerge_lora(self) -> None:
        """Drop the merged fp16 weight and return to the quantized path."""
        if not self.merged:
            raise RuntimeError("LoRA is not merged — nothing to unmerge")
        self.base_layer.merged_fp16_weight = None
        self.base_layer.merged_mode = False
        self.merged = False
        layer_ops.forget_casts(self.lora_A, self.lora_B)

    def get_trainable_params(self) -> int:
        """Total number of trainable parameters in the LoRA layer."""
        return sum(p.numel() for p in self.parameters() if p.requires_grad)

    def extra_repr(self) -> str:
        return f"r={self.r}, alpha={self.lora_alpha}, scaling={self.scaling:.4f}, merged={self.merged}"
