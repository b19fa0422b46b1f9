"""Merged-weight export (the reference's rocm_qlora/export/gguf_export.py):
dequantize every LoRALinear's base weight, add its adapter delta in fp16 and
save a Hugging Face-style fp16 state dict (safetensors or .pt) that llama.cpp
can convert to GGUF.  The per-layer merge runs on the GPU in one pass over
the codes (rq_merge_lora).  The reference's vLLM helpers are not part of
this package."""
from rocm_qlora.export.gguf_export import (
    estimate_gguf_size,
    get_gguf_conversion_instructions,
    merge_and_export_fp16,
)

__all__ = ["merge_and_export_fp16", "get_gguf_conversion_instructions", "estimate_gguf_size"]
