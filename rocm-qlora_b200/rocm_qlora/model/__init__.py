"""Model-level quantization orchestration for rocm-qlora."""
from rocm_qlora.model.quantize_model import quantize_model, enable_all_kernels

__all__ = ["quantize_model", "enable_all_kernels"]
