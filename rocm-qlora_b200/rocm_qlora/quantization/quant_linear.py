"""QuantLinear: a Linear layer whose weight is stored NF4 / INT8 quantized.

Same constructor, buffers, flags and methods as the reference
(rocm_qlora/quantization/quant_linear.py:16-200), so state_dicts and calling
code interchange.  ``forward`` runs the fused dequantize-and-multiply kernel
of the B200 library (decode GEMV or tcgen05 GEMM, chosen by shape); there is
no separate dequantize pass and no CPU path.
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rocm_qlora import _native as nat
from rocm_qlora.quantization.quant_ops import (
    quantize_int8, dequantize_int8,
    quantize_int4, dequantize_int4
)
from rocm_qlora.quantization import layer_ops


class QuantLinear(nn.Module):
    """A Linear layer that stores weights in quantized format and
    dequantizes them on the fly inside the matmul kernel."""

    def __init__(self, in_features: int, out_features: int, bits: int = 8, bias: bool = True,
                 block_size: int = 64):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.bits = bits
        self.block_size = block_size
        self.original_shape: Optional[Tuple[int, ...]] = (out_features, in_features)
        # buffers, not parameters: frozen, moved by .to(), saved in state_dict
        self.register_buffer("weight_quant", torch.empty(0, dtype=torch.int8 if bits == 8 else torch.uint8))
        self.register_buffer("weight_scales", torch.empty(0))
        self.register_buffer("weight_zeros", torch.zeros(1))  # reserved (asymmetric quantization)
        if bias:
            self.register_buffer("bias", torch.zeros(out_features))
        else:
            self.bias = None
        self.use_triton_kernel: bool = False  # kept for API compatibility; see enable_kernel()
        self.use_double_quant: bool = False
        self.register_buffer("merged_fp16_weight", None)
        self.merged_mode: bool = False

    @classmethod
    def from_linear(cls, linear: nn.Linear, bits: int = 8, block_size: int = 64) -> "QuantLinear":
        """Quantize an nn.Linear (weights flattened, blockwise) and delete its
        original weight and bias to reclaim memory."""
        instance = cls(in_features=linear.in_features, out_features=linear.out_features, bits=bits,
                       bias=linear.bias is not None, block_size=block_size)
        instance.original_shape = linear.weight.shape
        flat_weight = linear.weight.data.flatten()
        if bits == 8:
            q_weight, scales = quantize_int8(flat_weight, block_size=block_size)
        elif bits == 4:
            q_weight, scales = quantize_int4(flat_weight, block_size=block_size)
        else:
            raise ValueError(f"Unsupported bit depth: {bits}")
        instance.weight_quant = q_weight
        instance.weight_scales = scales
        if linear.bias is not None:
            instance.bias = linear.bias.data.clone()
        del linear.weight
        if linear.bias is not None:
            del linear.bias
        return instance

    def enable_kernel(self) -> bool:
        """Report whether the fused B200 kernels can run here (library built,
        sm_100 device present).  The forward pass always uses them; this only
        sets the compatibility flag the reference's callers read."""
        ok = nat.is_available()
        self.use_triton_kernel = ok
        return ok

    def enable_double_quant(self) -> bool:
        """Switch this layer to double-quantized scales (returns True)."""
        from rocm_qlora.quantization.double_quant import patch_quant_linear_for_double_quant

        class Wrapper(nn.Module):
            def __init__(self, layer):
                super().__init__()
                self.layer = layer

        return patch_quant_linear_for_double_quant(Wrapper(self)) > 0

    def dequantized_weight(self) -> torch.Tensor:
        """fp32 [out, in] weight exactly as the reference's dequantize_* calls
        return it (used by merge/export, not by forward)."""
        n = self.out_features * self.in_features
        if self.bits == 4 and self.use_double_quant:
            from rocm_qlora.quantization.double_quant import DoubleQuantState, double_dequantize
            return double_dequantize(DoubleQuantState(
                W_quant=self.weight_quant, c2=self.c2, c2_scales=self.c2_scales, blocksize_1=self.block_size,
                blocksize_2=self.blocksize_2, original_shape=self.original_shape, use_fp8_c2=self.use_fp8_c2))
        if self.bits == 8:
            w = dequantize_int8(self.weight_quant, self.weight_scales, block_size=self.block_size)
        else:
            w = dequantize_int4(self.weight_quant, self.weight_scales, block_size=self.block_size)
        return w.reshape(-1)[:n].reshape(self.original_shape)

    _QUANT_BUFFERS = ("weight_quant", "weight_scales", "c2", "c2_scales")

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        """Loads quantized buffers whatever this module held before: a layer
        built unquantized (empty buffers) or quantized with another shape
        takes the checkpoint's shapes and dtypes, and a checkpoint carrying
        double-quantized scales (c2, c2_scales) switches the layer to them,
        so a state dict written by the reference loads into a fresh layer."""
        dq_keys = [prefix + k in state_dict for k in ("c2", "c2_scales")]
        if all(dq_keys):
            c2 = state_dict[prefix + "c2"]
            for k in ("c2", "c2_scales"):
                if k not in self._buffers:
                    self.register_buffer(k, torch.empty(0, device=self.weight_quant.device))
            self.use_double_quant = True
            self.use_fp8_c2 = c2.dtype != torch.int8
            self.blocksize_2 = getattr(self, "blocksize_2", 256)
        for k in self._QUANT_BUFFERS:
            t = state_dict.get(prefix + k)
            cur = self._buffers.get(k)
            if isinstance(t, torch.Tensor) and isinstance(cur, torch.Tensor) and (
                    cur.shape != t.shape or cur.dtype != t.dtype):
                self._buffers[k] = torch.empty(t.shape, dtype=t.dtype, device=cur.device)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def weight_view(self) -> layer_ops.WeightView:
        """The C ABI's view of the quantized buffers, rebuilt only when a
        buffer was replaced (module moves, new tensors) or written in place
        (version counter), or the format flags changed."""
        bufs = (self.weight_quant, getattr(self, "weight_scales", None), getattr(self, "c2", None),
                getattr(self, "c2_scales", None))
        if any(isinstance(t, torch.Tensor) and t.is_inference() for t in bufs):
            # inference tensors carry no version counter: no cache
            return layer_ops.weight_view(self)
        key = (self.bits, self.block_size, getattr(self, "use_double_quant", False), getattr(self, "use_fp8_c2", True),
               tuple((t.data_ptr(), t._version, t.shape, t.dtype) if isinstance(t, torch.Tensor) else None
                     for t in bufs))
        c = self.__dict__.get("_weight_view_cache")
        if c is not None and c[0] == key:
            return c[1]
        wv = layer_ops.weight_view(self)
        self.__dict__["_weight_view_cache"] = (key, wv)
        return wv

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.merged_mode and self.merged_fp16_weight is not None:
            weight = self.merged_fp16_weight.to(x.dtype)
            bias = self.bias.to(x.dtype) if self.bias is not None else None
            return F.linear(x, weight, bias)
        if torch.is_grad_enabled() and x.requires_grad:
            return layer_ops.QuantLinearFunction.apply(x, self.weight_view(), self.bias)
        return layer_ops.quant_forward(x, self.weight_view(), self.bias)

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, bits={self.bits}, block_size={self.block_size}"
