"""Device description and kernel configuration (reference
rocm_qlora/kernels/kernel_config.py), for B200.

The reference picks Triton tile sizes per AMD architecture; here the tile
shapes are fixed by the sm_100a kernels and reported for information.
``is_triton_available`` keeps its name and returns whether the fused B200
kernels can run (there is no Triton in this build's compute path).
"""
from dataclasses import dataclass
from typing import Any, Dict

import torch

from rocm_qlora import _native as nat


@dataclass
class KernelConfig:
    BLOCK_M: int
    BLOCK_N: int
    BLOCK_K: int
    num_warps: int
    num_stages: int
    wavefront_size: int  # warp width: 32 on NVIDIA


# tcgen05 dequant-GEMM tile (M x N x K per CTA) and the decode GEMV layout
B200_GEMM_CONFIG = KernelConfig(BLOCK_M=128, BLOCK_N=256, BLOCK_K=64, num_warps=8, num_stages=4, wavefront_size=32)
TritonKernelConfig = KernelConfig  # name used by the reference's callers


def detect_gpu_arch() -> str:
    if not torch.cuda.is_available():
        return "unknown"
    major, minor = torch.cuda.get_device_capability(0)
    return f"sm_{major}{minor}"


def get_kernel_config() -> KernelConfig:
    return B200_GEMM_CONFIG


def is_triton_available() -> bool:
    """True when the fused B200 kernels are usable on this machine."""
    return nat.is_available()


def get_device_info() -> Dict[str, Any]:
    if not torch.cuda.is_available():
        return {"arch": "unknown", "compute_units": 0, "vram_gb": 0.0, "wavefront_size": 32,
                "triton_available": False, "native_kernels": False}
    props = torch.cuda.get_device_properties(0)
    return {
        "arch": detect_gpu_arch(),
        "compute_units": getattr(props, "multi_processor_count", 0),
        "vram_gb": props.total_memory / (1024 ** 3),
        "wavefront_size": 32,
        "triton_available": is_triton_available(),
        "native_kernels": nat.is_available(),
    }
