"""FP8 compute configuration and hardware detection (the reference's
rocm_qlora/fp8/fp8_config.py, same names, keys and defaults).

The reference gates FP8 behind ROCm 6.2 and CDNA3.  Here the gate is the
hardware this build runs on: a CUDA device with FP8 tensor cores (compute
capability 8.9 or newer; B200 is 10.0), the float8_e4m3fn / float8_e5m2
dtypes in torch, and torch._scaled_mm (the cuBLASLt FP8 GEMM).  NVIDIA FP8 is
the OCP format: e4m3fn (largest value 448) and e5m2, so get_fp8_dtype
returns those; the fnuz variants the reference prefers are AMD's and have no
tensor-core support on NVIDIA GPUs.
"""
from dataclasses import dataclass
from typing import Any, Dict

import torch


def _fp8_dtypes_available() -> bool:
    return hasattr(torch, "float8_e4m3fn") and hasattr(torch, "float8_e5m2")


def detect_fp8_support() -> Dict[str, Any]:
    """Whether FP8 GEMMs can run here; never raises (CPU-only hosts report
    False with the reason)."""
    info = {
        "fp8_supported": False,
        "rocm_version": "not ROCm",
        "arch": "unknown",
        "fp8_dtypes_available": _fp8_dtypes_available(),
        "transformer_engine_available": False,
        "reason": "",
    }
    if getattr(torch.version, "hip", None):
        info["rocm_version"] = torch.version.hip
    try:
        import transformer_engine.pytorch  # noqa: F401
        info["transformer_engine_available"] = True
    except Exception:
        pass
    cap = None
    try:
        if torch.cuda.is_available():
            cap = torch.cuda.get_device_capability()
            info["arch"] = f"sm_{cap[0]}{cap[1]}"
    except Exception:
        cap = None
    if not info["fp8_dtypes_available"]:
        info["reason"] = "FP8 dtypes unavailable in this PyTorch build"
    elif cap is None:
        info["reason"] = "No CUDA device: FP8 tensor cores required"
    elif cap < (8, 9):
        info["reason"] = f"Unsupported GPU architecture ({info['arch']}) - FP8 tensor cores need sm_89 or newer"
    elif not hasattr(torch, "_scaled_mm"):
        info["reason"] = "torch._scaled_mm (FP8 GEMM) unavailable in this PyTorch build"
    else:
        info["fp8_supported"] = True
        info["reason"] = "Supported"
    return info


@dataclass
class FP8Config:
    """Configuration for FP8 training (defaults as the reference's)."""
    enabled: bool = True
    forward_dtype: str = "e4m3"          # E4M3 for weights/activations
    backward_dtype: str = "e5m2"         # E5M2 for gradients
    use_transformer_engine: bool = True  # prefer TE if available
    fallback_dtype: torch.dtype = torch.bfloat16
    amax_history_len: int = 16
    amax_compute_algo: str = "max"       # "max" or "most_recent"


def get_fp8_dtype(format_str: str) -> torch.dtype:
    """torch dtype of an FP8 format name: "e4m3" -> float8_e4m3fn,
    "e5m2" -> float8_e5m2 (the formats NVIDIA tensor cores take)."""
    if format_str == "e4m3":
        if hasattr(torch, "float8_e4m3fn"):
            return torch.float8_e4m3fn
        raise RuntimeError("No FP8 E4M3 dtype available. Check PyTorch version.")
    if format_str == "e5m2":
        if hasattr(torch, "float8_e5m2"):
            return torch.float8_e5m2
        raise RuntimeError("No FP8 E5M2 dtype available. Check PyTorch version.")
    raise ValueError(f"Unknown FP8 format: {format_str}")


def get_fp8_recipe(config: FP8Config):
    """A TransformerEngine DelayedScaling recipe, or None without TE."""
    try:
        import transformer_engine.pytorch as te
        return te.recipe.DelayedScaling(amax_history_len=config.amax_history_len,
                                        amax_compute_algo=config.amax_compute_algo)
    except Exception:
        return None
