"""HuggingFace integration: the quantization config and the HfQuantizer
(the reference's rocm_qlora/hf_integration/__init__.py exports)."""
from rocm_qlora.hf_integration.config import RocmQLoraConfig
from rocm_qlora.hf_integration.quantizer import RocmQLoraQuantizer

__all__ = ["RocmQLoraConfig", "RocmQLoraQuantizer"]
