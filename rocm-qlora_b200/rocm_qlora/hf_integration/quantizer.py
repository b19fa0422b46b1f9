"""HuggingFace ``HfQuantizer`` for this build (the reference's
rocm_qlora/hf_integration/quantizer.py:27-94): the same class name, flags and
hooks, so a caller that builds ``RocmQLoraQuantizer(RocmQLoraConfig(...))`` and
runs its hooks around weight loading gets the same model structure.

* ``_process_model_before_weight_loading`` replaces the configured target
  Linear layers with ``LoRALinear(QuantLinear)`` through ``quantize_model``
  (the quantization itself runs on the B200 kernels).
* ``_process_model_after_weight_loading`` marks the quantized layers
  kernel-enabled (``enable_all_kernels``) when ``use_triton_kernels`` is set
  -- the flag keeps its name and selects the fused B200 kernels -- and prints
  the trainable / total parameter report.  ``use_flash_attention`` asks the
  reference to patch the model's attention; attention is not part of this
  build's quantized-layer path, so the flag is accepted and left unused.
* ``validate_environment`` never raises for missing hardware: it warns when
  no CUDA device or no B200 kernels are present (the reference warns about a
  missing GPU or ROCm), and raises ImportError for transformers < 4.40 as the
  reference does.
"""
from typing import List

import torch
import torch.nn as nn

from rocm_qlora import _native as nat
from rocm_qlora.model.quantize_model import enable_all_kernels, quantize_model

try:
    import transformers
    from transformers.quantizers.base import HfQuantizer
except ImportError:  # transformers absent: the class exists, constructing it says why it cannot work
    transformers = None

    class HfQuantizer:
        def __init__(self, quantization_config, **kwargs):
            raise ImportError("transformers >= 4.40 required for HF plugin. "
                              "Use quantize_model() directly instead.")


class RocmQLoraQuantizer(HfQuantizer):
    """Quantizer class for rocm-qlora."""
    requires_calibration: bool = False
    required_packages: List[str] = ["rocm_qlora"]

    def validate_environment(self, *args, **kwargs):
        """Check hardware and software requirements (warnings only for the
        hardware; an old transformers raises)."""
        if not torch.cuda.is_available():
            print("[rocm-qlora] WARNING: No GPU detected. The quantized layers need a B200 (sm_100) device.")
        elif not nat.is_available():
            print("[rocm-qlora] WARNING: B200 kernels unavailable on this device "
                  "(library not built or not an sm_100 GPU).")
        from packaging import version
        if version.parse(transformers.__version__) < version.parse("4.40.0"):
            raise ImportError(f"transformers >= 4.40.0 required for rocm-qlora plugin. "
                              f"Found {transformers.__version__}. Please upgrade.")

    def _process_model_before_weight_loading(self, model: nn.Module, **kwargs) -> nn.Module:
        """Replace the target Linear layers with QuantLinear + LoRALinear."""
        config = self.quantization_config
        return quantize_model(model, bits=config.bits, lora_r=config.lora_r, lora_alpha=config.lora_alpha,
                              lora_dropout=config.lora_dropout, target_modules=config.target_modules,
                              block_size=config.block_size)

    def _process_model_after_weight_loading(self, model: nn.Module, **kwargs) -> nn.Module:
        """Enable the fused kernels once the weights are in memory; report
        the parameter counts."""
        config = self.quantization_config
        if config.use_triton_kernels:
            enable_all_kernels(model)
        trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
        total = sum(p.numel() for p in model.parameters())
        print(f"[rocm-qlora] Model ready. Trainable: {trainable:,} / Total: {total:,}")
        return model

    def is_serializable(self, *args, **kwargs) -> bool:
        return True

    def is_trainable(self, model: nn.Module = None) -> bool:
        return True
