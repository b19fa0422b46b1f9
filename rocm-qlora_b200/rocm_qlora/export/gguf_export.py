"""fp16 export of a fine-tuned model, the first step towards GGUF.

Same functions, arguments and results as the reference's
rocm_qlora/export/gguf_export.py:
  * ``_export_dequant_layer(lora_linear)``: the layer's weight dequantized
    and its adapter delta added, both in fp16 (export/gguf_export.py:30-80:
    W.to(fp16) + ((B @ A) * scaling).to(fp16)).  Here it is one kernel pass
    over the codes (rq_merge_lora, mode RQ_MERGE_ROUND_EACH), with no fp32
    copy of the weight or of the delta in memory;
  * ``_build_export_state_dict(model)``: every parameter that is not a LoRA
    adapter in fp16, and for each LoRALinear its merged ``.weight`` (and
    ``.bias``) under the module's name, the Hugging Face layout;
  * ``merge_and_export_fp16(model, path, model_config=None)``: that state
    dict saved as safetensors (or torch .pt for other extensions), with an
    optional config.json beside it;
  * ``get_gguf_conversion_instructions`` / ``estimate_gguf_size``: the
    llama.cpp conversion steps and a size estimate per GGUF type.
"""
import json
import os
from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from rocm_qlora.lora.lora_layer import LoRALinear
from rocm_qlora.quantization import layer_ops
from rocm_qlora.quantization.quant_linear import QuantLinear


def _export_dequant_layer(lora_linear: nn.Module) -> torch.Tensor:
    """fp16 [out, in]: fp16(deq(W)) + fp16(B @ A * scaling), added in fp16."""
    if not isinstance(lora_linear, LoRALinear):
        raise TypeError(f"Expected LoRALinear, got {type(lora_linear)}")
    quant = lora_linear.base_layer
    if not isinstance(quant, QuantLinear):
        raise TypeError(f"Expected a QuantLinear base layer, got {type(quant)}")
    if quant.weight_quant.is_cuda:
        return layer_ops.merge_weight(quant.weight_view(), lora_linear.lora_A, lora_linear.lora_B,
                                      lora_linear.scaling, layer_ops.MERGE_ROUND_EACH, torch.float16)
    # buffers on the host: the same sums with the library's dequantization
    W = quant.dequantized_weight().to(torch.float16)
    delta = ((lora_linear.lora_B @ lora_linear.lora_A) * lora_linear.scaling).to(torch.float16)
    return W + delta


def _build_export_state_dict(model: nn.Module) -> Dict[str, torch.Tensor]:
    """Hugging Face-style fp16 state dict with the adapters merged."""
    state_dict: Dict[str, torch.Tensor] = {}
    for name, param in model.named_parameters():
        if "lora_A" not in name and "lora_B" not in name:
            state_dict[name] = param.data.cpu().to(torch.float16)
    for name, module in model.named_modules():
        if isinstance(module, LoRALinear):
            state_dict[f"{name}.weight"] = _export_dequant_layer(module).cpu()
            if module.base_layer.bias is not None:
                state_dict[f"{name}.bias"] = module.base_layer.bias.data.cpu().to(torch.float16)
    return state_dict


def merge_and_export_fp16(model: nn.Module, output_path: str,
                          model_config: Optional[Dict[str, Any]] = None) -> str:
    """Writes the merged fp16 weights to `output_path` (.safetensors, else a
    torch .pt file) and, if given, `model_config` as config.json in the same
    directory.  Returns the path."""
    model.eval()
    with torch.no_grad():
        state_dict = _build_export_state_dict(model)
        total = sum(v.numel() * v.element_size() for v in state_dict.values())
        print(f"[export] {len(state_dict)} tensors, {total / 1e9:.2f} GB in fp16")
        if output_path.endswith(".safetensors"):
            try:
                from safetensors.torch import save_file
                save_file({k: v.contiguous() for k, v in state_dict.items()}, output_path)
            except ImportError:
                torch.save(state_dict, output_path)
                print("[export] safetensors is not installed: wrote a torch file instead")
        else:
            torch.save(state_dict, output_path)
        if model_config is not None:
            with open(os.path.join(os.path.dirname(output_path), "config.json"), "w") as f:
                json.dump(model_config, f, indent=2)
        print(f"[export] wrote {output_path}")
    return output_path


def get_gguf_conversion_instructions(fp16_path: str, model_type: str = "llama") -> str:
    """Shell steps that turn the exported fp16 file into a GGUF model with
    llama.cpp's converter and run it (llama.cpp or Ollama)."""
    return (
        f"# 1. llama.cpp and its Python requirements\n"
        f"git clone https://github.com/ggerganov/llama.cpp && cd llama.cpp && pip install -r requirements.txt\n"
        f"# 2. fp16 weights ({model_type} architecture) to GGUF, Q4_K_M quantization\n"
        f"python convert_hf_to_gguf.py {fp16_path} --outtype q4_k_m --outfile model.gguf\n"
        f"# 3. run it\n"
        f"./llama-cli -m model.gguf -p \"Hello\" -n 128\n"
        f"# or with Ollama: a Modelfile holding 'FROM ./model.gguf', then\n"
        f"ollama create my-model -f Modelfile && ollama run my-model\n")


# average bits per parameter of the GGUF weight types (llama.cpp's formats)
_GGUF_BITS = {"q2_k": 2.6, "q3_k_m": 3.35, "q4_0": 4.0, "q4_k_m": 4.5, "q5_k_m": 5.5, "q6_k": 6.0, "q8_0": 8.0,
              "f16": 16.0, "f32": 32.0}


def estimate_gguf_size(num_params: int, quant_type: str = "q4_k_m") -> Dict[str, Any]:
    """Approximate GGUF file size: parameters x bits per parameter, plus 5 %
    for metadata (unknown types count as q4_k_m)."""
    bits = _GGUF_BITS.get(quant_type, 4.5)
    return {"num_params": num_params, "quant_type": quant_type,
            "estimated_size_gb": round(num_params * bits / 8 / 1e9 * 1.05, 2), "bits_per_param": bits}
