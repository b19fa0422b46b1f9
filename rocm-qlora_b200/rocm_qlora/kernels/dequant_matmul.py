"""Fused dequantize + matmul entry points (reference
rocm_qlora/kernels/dequant_matmul.py:356-376), on the B200 kernels.

``fused_dequant_nf4_matmul(x, w_packed, scales, bias, block_size)`` and the
INT8 twin compute ``F.linear(x, deq(W).to(x.dtype), bias)`` with autograd
(input gradient through the transposed-weight kernel).  ``w_packed`` may be
1-D or [N, K/2]; N is inferred from x's last dimension as in the reference.
"""
import torch

from rocm_qlora import _native as nat
from rocm_qlora.quantization import layer_ops


def _view(fmt, q, scales, N, K, block_size):
    return layer_ops.WeightView(fmt, q.reshape(-1) if fmt != nat.W_INT8_ROW else q.contiguous(),
                                scales.reshape(-1).contiguous(), None, None, N, K, block_size)


def fused_dequant_int8_matmul(x, w_int8, scales, bias=None, block_size=64):
    """F.linear(x, dequantize_int8(w_int8, scales).to(x.dtype), bias); w_int8 is [N, K]."""
    N, K = w_int8.shape
    per_row = scales.numel() == N and N * K // block_size != N
    fmt = nat.W_INT8_ROW if per_row else nat.W_INT8
    return layer_ops.QuantLinearFunction.apply(x, _view(fmt, w_int8, scales, N, K, block_size), bias)


def fused_dequant_nf4_matmul(x, w_packed, scales, bias=None, block_size=64):
    """F.linear(x, dequantize_int4(w_packed, scales).to(x.dtype), bias)."""
    K = x.shape[-1]
    N = w_packed.numel() * 2 // K
    return layer_ops.QuantLinearFunction.apply(x, _view(nat.W_NF4, w_packed, scales, N, K, block_size), bias)
