"""FP8 compute over quantized storage (the reference's rocm_qlora.fp8):
FP8 tensor-core GEMMs on GPUs that have them (B200: e4m3fn), the wrapped
layer unchanged elsewhere."""
from rocm_qlora.fp8.fp8_config import (
    FP8Config, detect_fp8_support, get_fp8_dtype, get_fp8_recipe,
)
from rocm_qlora.fp8.fp8_linear import (
    FP8LinearWrapper, enable_fp8_autocast, weight_fp8, wrap_model_for_fp8,
)

__all__ = [
    "detect_fp8_support", "FP8Config", "get_fp8_dtype", "get_fp8_recipe",
    "FP8LinearWrapper", "wrap_model_for_fp8", "enable_fp8_autocast", "weight_fp8",
]
