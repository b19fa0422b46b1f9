"""Seeded synthetic inputs for the BASELINE configurations.

Inputs are drawn on the CPU with ``torch.Generator().manual_seed(seed)`` in a
fixed order -- W, X, A, B, dY -- so every machine with the same torch build
produces the same bytes, independent of any device RNG.  Distributions:
W ~ N(0, sigma), X and dY ~ N(0, 1), A ~ U(-1/sqrt(K), 1/sqrt(K)),
B ~ N(0, 0.01).  Nothing here reads a dataset: the reference's benchmarks run
on synthetic tensors of these shapes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class LayerInputs:
    W: torch.Tensor           # [N, K] in w_dtype
    X: torch.Tensor           # [M, K] in x_dtype
    A: Optional[torch.Tensor]  # [r, K] fp32 (cast to x dtype by the layer)
    B: Optional[torch.Tensor]  # [N, r] fp32
    dY: Optional[torch.Tensor]  # [M, N] in x_dtype
    r: int
    alpha: int

    @property
    def scaling(self) -> float:
        return self.alpha / self.r


def layer_inputs(N: int, K: int, M: int, *, sigma: float = 0.02, r: int = 16, alpha: int = 32,
                 w_dtype=torch.bfloat16, x_dtype=torch.bfloat16, seed: int = 0,
                 with_dy: bool = False, lora: bool = True) -> LayerInputs:
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * sigma).to(w_dtype)
    X = torch.randn(M, K, generator=g).to(x_dtype)
    A = B = None
    if lora:
        bound = 1.0 / math.sqrt(K)
        A = (torch.rand(r, K, generator=g) * 2.0 - 1.0) * bound
        B = torch.randn(N, r, generator=g) * 0.01
    dY = torch.randn(M, N, generator=g).to(x_dtype) if with_dy else None
    return LayerInputs(W, X, A, B, dY, r, alpha)


# BASELINE.json configs, as (name, kwargs) pairs.
def config1() -> LayerInputs:
    """Config 1: CPU-runnable layer, fp32 W 4096x4096 N(0,0.02) seed 0, X 32x4096,
    r=16 alpha=32, B nonzero; NF4 bs64 fp32 scales, no double quant."""
    return layer_inputs(4096, 4096, 32, sigma=0.02, r=16, alpha=32,
                        w_dtype=torch.float32, x_dtype=torch.float32, seed=0)


DECODE_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008)]   # [N, K]
DECODE_M = [1, 4, 16]
PREFILL_M = [512, 2048, 8192]
SHAPES_70B = [(28672, 8192), (8192, 28672)]
