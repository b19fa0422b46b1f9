"""The HuggingFace quantizer (rocm_qlora.hf_integration.RocmQLoraQuantizer),
after the reference's tests/v3/test_hf_integration.py: its flags, the
environment check (no raise without a GPU), the after-loading hook, and --
on the B200, where the quantization runs -- the before-loading hook's layer
swap, with the swapped layer's output checked against the oracle of the
reference's eager path."""
import pytest
import torch
import torch.nn as nn

from oracle import oracle as orc
from tests.gpu_util import to_f32
from tests.test_gpu_linear import DTC, oracle_wdeq
from tests.tolerance import assert_matmul_close


class FakeModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(128, 128)
        self.v_proj = nn.Linear(128, 128)


def _quantizer(**kw):
    from rocm_qlora.hf_integration import RocmQLoraConfig, RocmQLoraQuantizer
    return RocmQLoraQuantizer(RocmQLoraConfig(**kw))


def test_quantizer_is_an_hf_quantizer_with_reference_flags():
    from transformers.quantizers.base import HfQuantizer
    q = _quantizer()
    assert isinstance(q, HfQuantizer)
    assert q.is_trainable() is True
    assert q.is_serializable() is True
    assert q.requires_calibration is False
    assert q.quantization_config.quant_method == "rocm_qlora"


def test_quantizer_validate_environment_no_crash():
    _quantizer().validate_environment()


def test_process_after_loading_returns_model(capsys):
    model = FakeModel()
    res = _quantizer()._process_model_after_weight_loading(model)
    assert res is model
    assert "Model ready. Trainable: 33,024 / Total: 33,024" in capsys.readouterr().out


@pytest.mark.gpu
def test_process_before_loading_replaces_linears():
    from rocm_qlora import _native as nat
    from rocm_qlora import LoRALinear, QuantLinear
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")
    torch.manual_seed(0)
    q = _quantizer(bits=8, lora_r=8, lora_alpha=16, target_modules=["q_proj"])
    model = FakeModel().cuda()
    model = q._process_model_before_weight_loading(model)
    assert isinstance(model.q_proj, LoRALinear) and isinstance(model.q_proj.base_layer, QuantLinear)
    assert isinstance(model.v_proj, nn.Linear)  # not a target
    model = q._process_model_after_weight_loading(model)
    assert model.q_proj.base_layer.use_triton_kernel
    lora = model.q_proj.cuda().eval()
    with torch.no_grad():
        lora.lora_B.normal_(0.0, 0.02)
        x = torch.randn(4, 128, device="cuda")
        y = lora(x)
    ql = lora.base_layer
    wdeq = oracle_wdeq(ql, 128, 128)
    y_ref = orc.loralinear_forward(to_f32(x), wdeq, ql.bias.float().cpu().numpy(),
                                   lora.lora_A.detach().float().cpu().numpy(),
                                   lora.lora_B.detach().float().cpu().numpy(), lora.scaling, DTC[torch.float32])
    assert_matmul_close(to_f32(y), y_ref, DTC[torch.float32])
