"""LoRA adapter layer for rocm-qlora."""
from rocm_qlora.lora.lora_layer import LoRALinear

__all__ = ["LoRALinear"]
