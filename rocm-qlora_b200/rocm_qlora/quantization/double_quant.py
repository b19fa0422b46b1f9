"""Double quantization of the NF4 block scales (QLoRA), on the B200 kernels.

Same API as the reference (rocm_qlora/quantization/double_quant.py): the
first-level absmax scales c1 (one per 64-block) are quantized again over
groups of 256 into one byte each (float8_e4m3fnuz, or int8 when fp8 is
unavailable) plus one fp32 absmax per group.  Codes, c2 and c2_scales are
bit-identical to the reference's.
"""
from dataclasses import dataclass
from typing import Any, Dict

import torch
import torch.nn as nn

from rocm_qlora import _native as nat
from rocm_qlora.quantization.quant_ops import dequantize_int4, quantize_int4


def _has_fp8() -> bool:
    """True when torch has an fp8 e4m3 dtype (reference double_quant.py:20-24)."""
    return hasattr(torch, 'float8_e4m3fnuz') or hasattr(torch, 'float8_e4m3fn')


def _get_fp8_dtype() -> torch.dtype:
    """float8_e4m3fnuz whenever torch has it, else float8_e4m3fn (reference
    double_quant.py:27-33).  The kernels encode e4m3fnuz."""
    if hasattr(torch, 'float8_e4m3fnuz'):
        return torch.float8_e4m3fnuz
    return torch.float8_e4m3fn


@dataclass
class DoubleQuantState:
    """Complete state for double-quantized weights."""
    W_quant: torch.Tensor        # NF4 packed uint8, shape [ceil(N*K/2)]
    c2: torch.Tensor             # second-level quantized scales (FP8 or INT8)
    c2_scales: torch.Tensor      # scales for c2, FP32, shape [ceil(num_blocks_1/blocksize_2)]
    blocksize_1: int = 64        # NF4 block size
    blocksize_2: int = 256       # second quantization block size
    original_shape: tuple = None  # (out_features, in_features)
    use_fp8_c2: bool = False     # whether c2 uses FP8 or INT8 fallback


def quantize_scales(c1: torch.Tensor, blocksize_2: int = 256, fp8: bool = True):
    """Second level of double_quantize: fp32 c1 -> (c2 bytes, c2_scales fp32)."""
    L = nat.lib()
    dev = nat.compute_device(c1)
    with torch.cuda.device(dev):
        c = nat.to_cuda(c1.reshape(-1).to(torch.float32))
        nb = c.numel()
        ng = (nb + blocksize_2 - 1) // blocksize_2
        c2 = torch.empty(ng * blocksize_2, dtype=torch.uint8, device=dev)
        c2s = torch.empty(ng, 1, dtype=torch.float32, device=dev)
        nat.check(L.rq_dq_quantize_scales(c.data_ptr(), nb, blocksize_2, int(fp8), c2.data_ptr(), c2s.data_ptr(),
                                          nat.stream_ptr(dev)), "rq_dq_quantize_scales")
        # the kernels encode float8_e4m3fnuz, the dtype the reference picks
        # whenever torch has it
        c2 = c2.view(torch.float8_e4m3fnuz) if fp8 else c2.view(torch.int8)
        return c2, c2s.squeeze()


def double_quantize(tensor: torch.Tensor, blocksize_1: int = 64, blocksize_2: int = 256) -> DoubleQuantState:
    """NF4-quantize `tensor`, then quantize its block scales (reference
    double_quant.py:46-97)."""
    original_shape = tensor.shape
    W_packed, c1 = quantize_int4(tensor, block_size=blocksize_1)
    use_fp8 = _has_fp8()
    c2, c2s = quantize_scales(c1.reshape(-1), blocksize_2, use_fp8)
    return DoubleQuantState(W_quant=W_packed, c2=c2.to(tensor.device), c2_scales=c2s.to(tensor.device),
                            blocksize_1=blocksize_1, blocksize_2=blocksize_2, original_shape=original_shape,
                            use_fp8_c2=use_fp8)


def double_dequantize(state: DoubleQuantState) -> torch.Tensor:
    """fp32 weight of shape original_shape (reference double_quant.py:99-122)."""
    L = nat.lib()
    home = state.W_quant.device
    numel = 1
    for d in state.original_shape:
        numel *= int(d)
    dev = nat.compute_device(state.W_quant, state.c2)
    with torch.cuda.device(dev):
        p = nat.to_cuda(state.W_quant.reshape(-1))
        c2 = nat.to_cuda(state.c2.reshape(-1)).view(torch.uint8)
        c2s = nat.to_cuda(state.c2_scales.reshape(-1).to(torch.float32))
        nb = (numel + state.blocksize_1 - 1) // state.blocksize_1
        if c2.numel() < nb or c2s.numel() * state.blocksize_2 < nb or 2 * p.numel() < numel:
            raise RuntimeError("double-quant state does not cover original_shape")
        out = torch.empty(numel, dtype=torch.float32, device=dev)
        nat.check(L.rq_dq_dequantize(p.data_ptr(), numel, c2.data_ptr(), c2s.data_ptr(), int(state.use_fp8_c2),
                                     state.blocksize_1, state.blocksize_2, out.data_ptr(), nat.F32,
                                     nat.stream_ptr(dev)), "rq_dq_dequantize")
        return out.reshape(state.original_shape).to(home)


def estimate_double_quant_savings(tensor: torch.Tensor, blocksize_1: int = 64, blocksize_2: int = 256
                                  ) -> Dict[str, Any]:
    """Memory of NF4 with fp32 scales vs. with double-quantized scales (pure
    arithmetic on sizes, reference double_quant.py:124-158)."""
    num_params = tensor.numel()
    num_blocks_1 = (num_params + blocksize_1 - 1) // blocksize_1
    num_blocks_2 = (num_blocks_1 + blocksize_2 - 1) // blocksize_2
    nf4_bytes = (num_params + 1) // 2
    c1_bytes_naive = num_blocks_1 * 4
    total_naive = nf4_bytes + c1_bytes_naive
    c2_bytes = num_blocks_1 * 1
    c2_scales_bytes = num_blocks_2 * 4
    total_dq = nf4_bytes + c2_bytes + c2_scales_bytes
    saved = total_naive - total_dq
    saved_pct = (saved / total_naive) * 100
    naive_bits = (total_naive * 8) / num_params
    dq_bits = (total_dq * 8) / num_params
    return {
        "without_dq_bytes": total_naive,
        "with_dq_bytes": total_dq,
        "saved_bytes": saved,
        "saved_pct": saved_pct,
        "bits_saved_per_param": naive_bits - dq_bits,
    }


def patch_quant_linear_for_double_quant(model: nn.Module) -> int:
    """Upgrade every 4-bit QuantLinear in `model` to double-quantized scales.

    As in the reference (double_quant.py:160-200): dequantize the weight to
    fp32, re-run NF4 quantization on it, quantize the resulting scales, keep
    the existing packed codes, register ``c2`` / ``c2_scales`` and replace
    ``weight_scales`` with an empty tensor.  Returns the number of layers."""
    from rocm_qlora.quantization.quant_linear import QuantLinear
    layers = [m for _, m in model.named_modules() if isinstance(m, QuantLinear) and m.bits == 4]
    for module in layers:
        W_fp = dequantize_int4(module.weight_quant, module.weight_scales, block_size=module.block_size)
        num_elements = module.out_features * module.in_features
        W_fp = W_fp[:num_elements].reshape(module.original_shape)
        state = double_quantize(W_fp, blocksize_1=module.block_size, blocksize_2=256)
        module.register_buffer("c2", state.c2)
        module.register_buffer("c2_scales", state.c2_scales)
        module.blocksize_2 = state.blocksize_2
        module.use_fp8_c2 = state.use_fp8_c2
        module.use_double_quant = True
        del module.weight_scales
        module.register_buffer("weight_scales", torch.empty(0, device=module.weight_quant.device))
    return len(layers)
