"""Standalone NF4 dequantization to bf16 (reference
rocm_qlora/kernels/nf4_dequant.py:81-115), on the B200 streaming kernel."""
from typing import Optional, Tuple

import torch

from rocm_qlora.quantization.quant_ops import NF4_VALUES, _dequantize_int4_as

NF4_TABLE = torch.tensor(NF4_VALUES, dtype=torch.float32)


def dequantize_nf4_triton(packed: torch.Tensor, scales: torch.Tensor, block_size: int = 64,
                          original_shape: Optional[Tuple[int, ...]] = None) -> torch.Tensor:
    """bf16 values T[code] * scale (rounded from fp32), optionally reshaped."""
    out = _dequantize_int4_as(packed, scales, block_size, torch.bfloat16)
    if original_shape:
        return out.view(original_shape)
    return out
