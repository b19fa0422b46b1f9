"""CPU oracle for rocm-qlora's quantize / dequantize / QuantLinear+LoRA path.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the cpu_baseline / reference legs of ``bench.py`` as the checker.  The
product package (``rocm-qlora_b200/rocm_qlora``) never imports it.

Byte and integer arithmetic (codes, scales, fp8 second-level scales) runs in
``rq_oracle.c`` (compiled by ``oracle/build.py`` into ``oracle/_build``).
The matmul legs are numpy restatements of the reference's eager path:

* ``quantlinear_forward``  rocm_qlora/quantization/quant_linear.py:182-197
  (dequantize -> ``.to(x.dtype)`` -> ``F.linear``),
* ``loralinear_forward``   rocm_qlora/lora/lora_layer.py:51-70
  (``base + ((x @ A.T) @ B.T) * scaling``, every product rounded to x.dtype),
* ``loralinear_dx``        the autograd of the two above with a frozen base.

Matmuls accumulate in float64 and round once per torch op, so they differ
from any fp32-accumulating implementation only by summation order.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

from . import build as _build

F32, BF16, F16 = 0, 1, 2
_NP_OF = {F32: np.float32, BF16: np.uint16, F16: np.uint16}

_lib = None


def lib() -> ctypes.CDLL:
    """Load (building first if needed) the compiled C restatement."""
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_nf4_quantize.argtypes = [P, I, I64, I, P, P]
        L.orc_nf4_quantize.restype = I64
        L.orc_nf4_dequantize.argtypes = [P, P, I, I64, I, P]
        L.orc_int8_quantize.argtypes = [P, I, I64, I, P, P]
        L.orc_int8_quantize.restype = I64
        L.orc_int8_quantize_rows.argtypes = [P, I, I64, I64, P, P]
        L.orc_int8_dequantize.argtypes = [P, P, I, I64, I, I64, I64, P]
        L.orc_dq_second_level.argtypes = [P, I64, I, I, P, P]
        L.orc_dq_second_level.restype = I64
        L.orc_dq_first_level.argtypes = [P, P, I64, I, I, P]
        L.orc_nf4_table.argtypes = [P]
        L.orc_f32_to_e4m3fnuz.argtypes = [ctypes.c_float]
        L.orc_f32_to_e4m3fnuz.restype = ctypes.c_uint8
        L.orc_e4m3fnuz_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3fnuz_to_f32.restype = ctypes.c_float
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ------------------------------------------------------------------ dtypes
# bf16 / f16 arrays are carried as uint16 bit patterns (numpy has no bf16).

def bf16_bits_to_f32(u: np.ndarray) -> np.ndarray:
    return (u.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    out = ((u + bias) >> 16).astype(np.uint16)
    out[np.isnan(f)] = 0x7FC0
    return out


def round_bf16(f: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 -> fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(f))


def f16_bits_to_f32(u: np.ndarray) -> np.ndarray:
    return u.astype(np.uint16).view(np.float16).astype(np.float32)


def round_to(f: np.ndarray, dtype: int) -> np.ndarray:
    f = np.asarray(f, dtype=np.float32)
    if dtype == BF16:
        return round_bf16(f)
    if dtype == F16:
        return f.astype(np.float16).astype(np.float32)
    return f


def to_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == BF16:
        return bf16_bits_to_f32(a)
    if dtype == F16:
        return f16_bits_to_f32(a)
    return np.asarray(a, dtype=np.float32)


def nf4_table() -> np.ndarray:
    t = np.zeros(16, np.float32)
    lib().orc_nf4_table(_ptr(t))
    return t


# ---------------------------------------------------------- quantization

def nf4_quantize(x: np.ndarray, dtype: int, block_size: int = 64) -> Tuple[np.ndarray, np.ndarray]:
    """quantize_int4 (quant_ops.py:80-126): (packed uint8, scales in x's dtype)."""
    x = np.ascontiguousarray(x.reshape(-1))
    n = x.size
    nb = (n + block_size - 1) // block_size
    packed = np.zeros(nb * block_size // 2, np.uint8)
    scales = np.zeros(nb, _NP_OF[dtype])
    r = lib().orc_nf4_quantize(_ptr(x), dtype, n, block_size, _ptr(packed), _ptr(scales))
    if r < 0:
        raise ValueError(f"unsupported block size {block_size}")
    return packed, scales


def nf4_dequantize(packed: np.ndarray, scales: np.ndarray, sdtype: int, block_size: int = 64) -> np.ndarray:
    """dequantize_int4 (quant_ops.py:128-150): fp32 [2*len(packed)]."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales)
    out = np.zeros(packed.size * 2, np.float32)
    lib().orc_nf4_dequantize(_ptr(packed), _ptr(scales), sdtype, packed.size, block_size, _ptr(out))
    return out


def int8_quantize(x: np.ndarray, dtype: int, block_size: int = 64) -> Tuple[np.ndarray, np.ndarray]:
    """quantize_int8 blockwise (quant_ops.py:36-53)."""
    x = np.ascontiguousarray(x.reshape(-1))
    n = x.size
    nb = (n + block_size - 1) // block_size
    q = np.zeros(nb * block_size, np.int8)
    scales = np.zeros(nb, _NP_OF[dtype])
    lib().orc_int8_quantize(_ptr(x), dtype, n, block_size, _ptr(q), _ptr(scales))
    return q, scales


def int8_quantize_rows(x: np.ndarray, dtype: int) -> Tuple[np.ndarray, np.ndarray]:
    """quantize_int8(per_channel=True) (quant_ops.py:28-35) of a [rows, cols] weight."""
    x = np.ascontiguousarray(x)
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int8)
    scales = np.zeros(rows, _NP_OF[dtype])
    lib().orc_int8_quantize_rows(_ptr(x), dtype, rows, cols, _ptr(q), _ptr(scales))
    return q, scales


def int8_dequantize(q: np.ndarray, scales: np.ndarray, sdtype: int, block_size: int = 64,
                    rows: int = 0, cols: int = 0) -> np.ndarray:
    """dequantize_int8 (quant_ops.py:55-78); rows>0 selects per-channel scales."""
    q = np.ascontiguousarray(q.reshape(-1), dtype=np.int8)
    scales = np.ascontiguousarray(scales)
    out = np.zeros(q.size, np.float32)
    lib().orc_int8_dequantize(_ptr(q), _ptr(scales), sdtype, q.size, block_size, rows, cols, _ptr(out))
    return out


def dq_second_level(c1: np.ndarray, blocksize_2: int = 256, fp8: bool = True) -> Tuple[np.ndarray, np.ndarray]:
    """Second level of double_quantize (double_quant.py:58-97)."""
    c1 = np.ascontiguousarray(c1, dtype=np.float32)
    nb = c1.size
    ng = (nb + blocksize_2 - 1) // blocksize_2
    c2 = np.zeros(ng * blocksize_2, np.uint8)
    c2s = np.zeros(ng, np.float32)
    lib().orc_dq_second_level(_ptr(c1), nb, blocksize_2, int(fp8), _ptr(c2), _ptr(c2s))
    return c2, c2s


def dq_first_level(c2: np.ndarray, c2s: np.ndarray, nb: int, blocksize_2: int = 256, fp8: bool = True) -> np.ndarray:
    """c1' = c2 * c2_scales (double_quant.py:103-115), truncated to nb."""
    c2 = np.ascontiguousarray(c2, dtype=np.uint8)
    c2s = np.ascontiguousarray(c2s, dtype=np.float32).reshape(-1)
    c1 = np.zeros(nb, np.float32)
    lib().orc_dq_first_level(_ptr(c2), _ptr(c2s), nb, blocksize_2, int(fp8), _ptr(c1))
    return c1


def enable_double_quant(packed: np.ndarray, scales: np.ndarray, sdtype: int, n_elems: int,
                        block_size: int = 64, fp8: bool = True):
    """QuantLinear.enable_double_quant (double_quant.py:174-196): dequantize to
    fp32, re-run quantize_int4 on the fp32 weight, then quantize its scales.
    Returns (c2, c2_scales); the packed codes stay as they are."""
    w = nf4_dequantize(packed, scales, sdtype, block_size)[:n_elems]
    _, c1 = nf4_quantize(w, F32, block_size)
    return dq_second_level(c1, 256, fp8)


def double_dequantize(packed: np.ndarray, c2: np.ndarray, c2s: np.ndarray, n_elems: int,
                      block_size: int = 64, fp8: bool = True) -> np.ndarray:
    """double_dequantize (double_quant.py:99-122): fp32 [n_elems]."""
    nb = (n_elems + block_size - 1) // block_size
    c1 = dq_first_level(c2, c2s, nb, 256, fp8)
    return nf4_dequantize(packed, c1, F32, block_size)[:n_elems]


# -------------------------------------------------------------- matmuls

def _mm(a: np.ndarray, b_t: np.ndarray) -> np.ndarray:
    """a @ b_t.T accumulated in float64."""
    return a.astype(np.float64) @ b_t.astype(np.float64).T


def quantlinear_forward(x: np.ndarray, w_deq: np.ndarray, bias: Optional[np.ndarray], dtype: int) -> np.ndarray:
    """QuantLinear.forward eager branch (quant_linear.py:191-197).

    x: fp32 values already representable in ``dtype``; w_deq: fp32 [N, K]
    (output of a dequantize_*); returns fp32 values representable in dtype."""
    w = round_to(w_deq, dtype)
    acc = _mm(x, w)
    if bias is not None:
        acc = acc + round_to(bias, dtype).astype(np.float64)
    return round_to(acc.astype(np.float32) if dtype == F32 else acc, dtype)


def lora_delta(x: np.ndarray, A: np.ndarray, B: np.ndarray, scaling: float, dtype: int) -> np.ndarray:
    """((x @ A.T) @ B.T) * scaling with the per-op roundings of lora_layer.py:67."""
    t = round_to(_mm(x, round_to(A, dtype)), dtype)
    u = round_to(_mm(t, round_to(B, dtype)), dtype)
    return round_to(u * np.float32(scaling), dtype)


def loralinear_forward(x, w_deq, bias, A, B, scaling, dtype) -> np.ndarray:
    """LoRALinear.forward in eval mode (lora_layer.py:51-70)."""
    base = quantlinear_forward(x, w_deq, bias, dtype)
    if A is None or B is None:
        return base
    return round_to(base + lora_delta(x, A, B, scaling, dtype), dtype)


def loralinear_dx(dy: np.ndarray, w_deq: np.ndarray, A, B, scaling, dtype) -> np.ndarray:
    """dX of LoRALinear.forward: dY @ W + s * (dY @ B) @ A (autograd of
    F.linear with a frozen weight plus the adapter product), each torch op
    rounded to dtype: grad of ``u*s`` is ``dy*s``, then ``@ B`` then ``@ A``."""
    w = round_to(w_deq, dtype)
    base = round_to(dy.astype(np.float64) @ w.astype(np.float64), dtype)
    if A is None or B is None:
        return base
    g = round_to(dy * np.float32(scaling), dtype)
    gt = round_to(g.astype(np.float64) @ round_to(B, dtype).astype(np.float64), dtype)
    ga = round_to(gt.astype(np.float64) @ round_to(A, dtype).astype(np.float64), dtype)
    return round_to(base + ga, dtype)
