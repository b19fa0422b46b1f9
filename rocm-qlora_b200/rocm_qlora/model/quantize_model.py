"""Model-level orchestration: swap nn.Linear layers for LoRALinear(QuantLinear).

Same API and replacement rules as the reference
(rocm_qlora/model/quantize_model.py:19-142): the model is frozen, every
nn.Linear whose qualified name ends with one of ``target_modules`` and whose
in/out features are both >= 64 is quantized (the original weight is freed)
and wrapped with a LoRA adapter.  Quantization runs on the B200 kernels.
"""
import logging
from typing import List, Tuple

import torch.nn as nn

from rocm_qlora.quantization.quant_linear import QuantLinear
from rocm_qlora.lora.lora_layer import LoRALinear

logger = logging.getLogger("rocm_qlora.quantize_model")


def _get_parent_and_attr(model: nn.Module, full_name: str) -> Tuple[nn.Module, str]:
    """(parent module, attribute name) of a dotted module path."""
    parts = full_name.split(".")
    parent = model
    for p in parts[:-1]:
        parent = getattr(parent, p)
    return parent, parts[-1]


def _summary(model: nn.Module, bits: int) -> None:
    total = sum(p.numel() for p in model.parameters())
    trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
    quant = [m for m in model.modules() if isinstance(m, QuantLinear)]
    qbytes = sum(m.weight_quant.numel() * m.weight_quant.element_size()
                 + m.weight_scales.numel() * m.weight_scales.element_size() for m in quant)
    qparams = sum(m.in_features * m.out_features for m in quant)
    pct = (trainable / total) * 100 if total > 0 else 0
    print("\n--- Model Quantization Summary ---")
    print(f"Quantized layers: {len(quant)} ({bits}-bit, {qparams:,} weights in {qbytes / 2**30:.4f} GiB)")
    print(f"Total Parameters: {total:,}")
    print(f"Trainable Parameters: {trainable:,} ({pct:.4f}%)")
    if qparams:
        print(f"Quantized weights vs fp16: {100 * (1 - qbytes / (2 * qparams)):.2f}% smaller")
    print("----------------------------------\n")


def quantize_model(model: nn.Module, bits: int = 8, lora_r: int = 8, lora_alpha: int = 16,
                   lora_dropout: float = 0.05, target_modules: List[str] = ["q_proj", "v_proj"],
                   block_size: int = 64) -> nn.Module:
    """Replace target Linear layers with LoRALinear(QuantLinear) and return the model."""
    if bits not in [4, 8]:
        raise ValueError(f"Invalid bit-depth: {bits}. Only 4 and 8 bits are supported.")
    model.requires_grad_(False)
    replacements = []
    for name, module in model.named_modules():
        if isinstance(module, nn.Linear) and any(name.endswith(t) for t in target_modules):
            if min(module.in_features, module.out_features) < 64:
                logger.warning(f"Skipping layer '{name}' because it is too small "
                               f"({module.in_features}x{module.out_features} < 64)")
                continue
            parent, attr = _get_parent_and_attr(model, name)
            replacements.append((parent, attr, module))
    for parent, child_attr, original_linear in replacements:
        ql = QuantLinear.from_linear(original_linear, bits=bits, block_size=block_size)
        setattr(parent, child_attr, LoRALinear(ql, r=lora_r, lora_alpha=lora_alpha, lora_dropout=lora_dropout))
    _summary(model, bits)
    return model


def enable_all_kernels(model: nn.Module) -> int:
    """Mark every QuantLinear (bare or inside a LoRALinear) as kernel-enabled;
    returns how many report the B200 kernels available."""
    enabled = 0
    for _, module in model.named_modules():
        target = None
        if isinstance(module, QuantLinear):
            target = module
        elif hasattr(module, "base_layer") and isinstance(module.base_layer, QuantLinear):
            target = module.base_layer
        if target is not None and target.enable_kernel():
            enabled += 1
    return enabled
