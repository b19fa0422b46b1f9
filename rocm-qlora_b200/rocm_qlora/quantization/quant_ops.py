"""NF4 and INT8 blockwise quantization on the B200 kernels.

Same functions, arguments, return shapes and dtypes as the reference
(rocm_qlora/quantization/quant_ops.py): blocks of ``block_size`` consecutive
elements of the flattened tensor, zero padded at the end; one absmax scale
per block kept in the input dtype; NF4 codes packed two per byte with the
even element in the low nibble.  Results are bit-identical to the
reference's (checked against its own outputs in tests/golden).
"""
from typing import Tuple

import torch

from rocm_qlora import _native as nat

# NF4 levels (quant_ops.py:10-15 of the reference)
NF4_VALUES = [
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0
]


def _squeeze_like_reference(scales_col: torch.Tensor) -> torch.Tensor:
    # the reference returns `scales.squeeze()` of a [nb, 1] tensor
    return scales_col.view(-1, 1).squeeze()


def quantize_int8(tensor: torch.Tensor, block_size: int = 64, per_channel: bool = False
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (int8_tensor, scales); scales are [num_blocks] or [out_channels]
    (reference quant_ops.py:17-53)."""
    L = nat.lib()
    home = tensor.device
    dev = nat.compute_device(tensor)
    dt = nat.dtype_code(tensor.dtype)
    with torch.cuda.device(dev):
        x = nat.to_cuda(tensor)
        st = nat.stream_ptr(dev)
        if per_channel:
            if x.dim() != 2:
                raise ValueError("per_channel quantization expects a 2-D [out, in] weight")
            rows, cols = x.shape
            q = torch.empty(rows, cols, dtype=torch.int8, device=dev)
            s = torch.empty(rows, 1, dtype=tensor.dtype, device=dev)
            nat.check(L.rq_int8_quantize_rows(x.data_ptr(), dt, rows, cols, q.data_ptr(), s.data_ptr(), st),
                      "rq_int8_quantize_rows")
            return q.to(home), s.squeeze().to(home)
        n = x.numel()
        nb = (n + block_size - 1) // block_size
        q = torch.empty(nb * block_size, dtype=torch.int8, device=dev)
        s = torch.empty(nb, 1, dtype=tensor.dtype, device=dev)
        nat.check(L.rq_int8_quantize(x.data_ptr(), dt, n, block_size, q.data_ptr(), s.data_ptr(), st),
                  "rq_int8_quantize")
        return q.to(home), _squeeze_like_reference(s).to(home)


def dequantize_int8(int8_tensor: torch.Tensor, scales: torch.Tensor, block_size: int = 64) -> torch.Tensor:
    """fp32 values q * scale, per-channel when int8_tensor is 2-D with one
    scale per row (reference quant_ops.py:55-78)."""
    L = nat.lib()
    home = int8_tensor.device
    dev = nat.compute_device(int8_tensor, scales)
    per_channel = int8_tensor.dim() == 2 and scales.numel() == int8_tensor.size(0)
    with torch.cuda.device(dev):
        q = nat.to_cuda(int8_tensor)
        s = nat.to_cuda(scales)
        out = torch.empty(q.numel(), dtype=torch.float32, device=dev)
        cols = q.size(1) if per_channel else 0
        if not per_channel and q.numel() % block_size:
            raise RuntimeError(f"shape '[-1, {block_size}]' is invalid for input of size {q.numel()}")
        if not per_channel and s.numel() * block_size < q.numel():
            raise RuntimeError(f"{s.numel()} scales do not cover {q.numel()} values in blocks of {block_size}")
        nat.check(L.rq_int8_dequantize(q.data_ptr(), q.numel(), s.data_ptr(), nat.dtype_code(s.dtype), block_size,
                                       cols, out.data_ptr(), nat.F32, nat.stream_ptr(dev)), "rq_int8_dequantize")
        if int8_tensor.dim() == 2:
            out = out.view(int8_tensor.shape)
        return out.to(home)


def quantize_int4(tensor: torch.Tensor, block_size: int = 64) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (packed_uint8, scales): NF4 codes two per byte (reference
    quant_ops.py:80-126)."""
    L = nat.lib()
    home = tensor.device
    dev = nat.compute_device(tensor)
    dt = nat.dtype_code(tensor.dtype)
    if block_size < 2 or block_size % 2:
        raise ValueError(f"block_size must be even, got {block_size}")
    with torch.cuda.device(dev):
        x = nat.to_cuda(tensor)
        n = x.numel()
        nb = (n + block_size - 1) // block_size
        packed = torch.empty(nb * block_size // 2, dtype=torch.uint8, device=dev)
        s = torch.empty(nb, 1, dtype=tensor.dtype, device=dev)
        nat.check(L.rq_nf4_quantize(x.data_ptr(), dt, n, block_size, packed.data_ptr(), s.data_ptr(),
                                    nat.stream_ptr(dev)), "rq_nf4_quantize")
        return packed.to(home), _squeeze_like_reference(s).to(home)


def dequantize_int4(packed: torch.Tensor, scales: torch.Tensor, block_size: int = 64) -> torch.Tensor:
    """fp32 [2 * packed.numel()] values T[code] * scale (reference
    quant_ops.py:128-150)."""
    return _dequantize_int4_as(packed, scales, block_size, torch.float32)


def _dequantize_int4_as(packed: torch.Tensor, scales: torch.Tensor, block_size: int, out_dtype: torch.dtype
                        ) -> torch.Tensor:
    L = nat.lib()
    home = packed.device
    dev = nat.compute_device(packed, scales)
    with torch.cuda.device(dev):
        p = nat.to_cuda(packed.reshape(-1))
        s = nat.to_cuda(scales.reshape(-1))
        if s.numel() * block_size < 2 * p.numel():
            raise RuntimeError(f"{s.numel()} scales do not cover {2 * p.numel()} values in blocks of {block_size}")
        out = torch.empty(2 * p.numel(), dtype=out_dtype, device=dev)
        nat.check(L.rq_nf4_dequantize(p.data_ptr(), p.numel(), s.data_ptr(), nat.dtype_code(s.dtype), block_size,
                                      out.data_ptr(), nat.dtype_code(out_dtype), nat.stream_ptr(dev)),
                  "rq_nf4_dequantize")
        return out.to(home)
