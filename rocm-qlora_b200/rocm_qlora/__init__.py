"""rocm-qlora, B200 build: the QLoRA hot path -- NF4/INT8 blockwise
quantization with optional double-quantized scales, and the fused
QuantLinear + LoRA layer (forward and input gradient) -- on hand-written
sm_100a kernels behind a C ABI (include/rq_b200.h).

The public names of the reference package's quantization, kernels, lora and
model layers are kept, so code written against rocm_qlora runs unchanged.
"""
import os

from rocm_qlora.quantization.quant_linear import QuantLinear
from rocm_qlora.lora.lora_layer import LoRALinear
from rocm_qlora.model.quantize_model import quantize_model, enable_all_kernels
from rocm_qlora.kernels import (
    fused_dequant_int8_matmul, fused_dequant_nf4_matmul,
    get_device_info, is_triton_available,
)
from rocm_qlora.hf_integration import RocmQLoraConfig

__version__ = "5.0.0+b200"

__all__ = [
    "quantize_model", "QuantLinear", "LoRALinear", "enable_all_kernels",
    "fused_dequant_int8_matmul", "fused_dequant_nf4_matmul",
    "get_device_info", "is_triton_available",
    "RocmQLoraConfig",
    "__version__",
]
