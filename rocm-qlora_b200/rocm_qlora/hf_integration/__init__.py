"""HuggingFace integration (config only in this build)."""
from rocm_qlora.hf_integration.config import RocmQLoraConfig

__all__ = ["RocmQLoraConfig"]
