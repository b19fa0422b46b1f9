"""FP8 compute over quantized storage (rocm_qlora.fp8), after the reference's
tests/v4/test_fp8.py: detection, configuration, wrapping and the fallback on
hosts without FP8 tensor cores run on the CPU; the native path runs on the
B200 against a torch restatement of the reference's native forward
(fp8_linear.py:27-39, 98-114): the e4m3fn weight bit for bit, the output
bit for bit (the same _scaled_mm call on the same operands), grad_x within
the matmul tolerance.
"""
import os
from unittest import mock

import numpy as np
import pytest
import torch
import torch.nn as nn

from rocm_qlora import LoRALinear, QuantLinear
from rocm_qlora.fp8 import (FP8Config, FP8LinearWrapper, detect_fp8_support, enable_fp8_autocast, get_fp8_dtype,
                            get_fp8_recipe, wrap_model_for_fp8)

KEYS = ["fp8_supported", "rocm_version", "arch", "fp8_dtypes_available", "transformer_engine_available", "reason"]


def test_detect_fp8_returns_dict_with_all_keys():
    res = detect_fp8_support()
    assert isinstance(res, dict)
    assert all(k in res for k in KEYS)
    assert isinstance(res["reason"], str) and res["reason"]


def test_detect_fp8_false_without_fp8_tensor_cores():
    res = detect_fp8_support()
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() < (8, 9):
        assert res["fp8_supported"] is False


def test_fp8_config_defaults_and_dtypes():
    c = FP8Config()
    assert c.forward_dtype == "e4m3" and c.backward_dtype == "e5m2" and c.enabled
    assert get_fp8_dtype("e4m3") == torch.float8_e4m3fn
    assert get_fp8_dtype("e5m2") == torch.float8_e5m2
    with pytest.raises(ValueError):
        get_fp8_dtype("e3m4")


def test_get_fp8_recipe_none_without_te():
    with mock.patch.dict("sys.modules", {"transformer_engine": None}):
        assert get_fp8_recipe(FP8Config()) is None


def _tiny_lora(n=32, k=32):
    ql = QuantLinear(k, n)
    ql.weight_quant = torch.zeros(n * k, dtype=torch.int8)
    ql.weight_scales = torch.ones(n * k // 64)
    return LoRALinear(ql)


def test_wrapper_backend_bf16_without_fp8():
    w = FP8LinearWrapper(_tiny_lora())
    if not detect_fp8_support()["fp8_supported"]:
        assert w.backend == "bf16"
    assert "backend=" in w.extra_repr()
    assert FP8LinearWrapper(_tiny_lora(), FP8Config(enabled=False)).backend == "bf16"


def test_wrap_model_status_and_env():
    os.environ.pop("TORCH_NCCL_HIGH_PRIORITY", None)
    model = nn.Sequential(LoRALinear(QuantLinear(4, 4)))
    res, info = wrap_model_for_fp8(model)
    assert isinstance(res, nn.Module) and isinstance(info, dict)
    assert all(k in info for k in ["enabled", "backend", "layers_wrapped", "reason"])
    if not detect_fp8_support()["fp8_supported"]:
        assert info["enabled"] is False and info["reason"]
        assert "TORCH_NCCL_HIGH_PRIORITY" not in os.environ


def test_enable_fp8_autocast_is_a_context():
    ctx = enable_fp8_autocast(nn.Linear(4, 4))
    assert hasattr(ctx, "__enter__") and hasattr(ctx, "__exit__")
    with enable_fp8_autocast(nn.Linear(4, 4)):
        pass


# ------------------------------------------------------------------- GPU

def _gpu_layer(N, K, bits, dq, bias, seed, r=16):
    g = torch.Generator().manual_seed(seed)
    lin = nn.Linear(K, N, bias=bias, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        if bias:
            lin.bias.copy_(torch.randn(N, generator=g) * 0.1)
    ql = QuantLinear.from_linear(lin.cuda(), bits=bits)
    if dq:
        ql.enable_double_quant()
    lora = LoRALinear(ql, r=r, lora_alpha=2 * r).cuda()
    with torch.no_grad():
        lora.lora_B.copy_(torch.randn(N, r, generator=g).cuda() * 0.01)
    return lora


def _ref_native(lora, x):
    """The reference's native FP8 forward restated with torch ops on the
    dequantized weight (fp32 from the library's dequantize, as its
    dequantize_* returns), and its e4m3 weight."""
    ql = lora.base_layer
    w = ql.dequantized_weight().to(x.dtype)
    f8 = torch.float8_e4m3fn
    w_scale = torch.tensor(w.abs().max().item() / 448.0, dtype=torch.float32, device=x.device)
    w_f8 = (w / w_scale).to(f8)
    x2 = x.reshape(-1, x.shape[-1])
    x_scale = torch.tensor(x2.abs().max().item() / 448.0, dtype=torch.float32, device=x.device)
    x_f8 = (x2 / x_scale).to(f8)
    out = torch._scaled_mm(x_f8, w_f8.t(), scale_a=x_scale, scale_b=w_scale, out_dtype=x.dtype)
    out = out.reshape(*x.shape[:-1], -1)
    if ql.bias is not None:
        out = out + ql.bias.to(x.dtype)
    lora_out = x @ lora.lora_A.t().to(x.dtype) @ lora.lora_B.t().to(x.dtype) * lora.scaling
    return out + lora_out.to(out.dtype), w, w_f8, w_scale


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,bits,dq,bias", [(1024, 4096, 4, True, False), (768, 2048, 4, False, True),
                                              (512, 1024, 8, False, False)])
def test_native_fp8_forward_backward(N, K, bits, dq, bias):
    from rocm_qlora import _native as nat
    from rocm_qlora.fp8 import weight_fp8
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")
    lora = _gpu_layer(N, K, bits, dq, bias, seed=N + K + bits).eval()
    wrap = FP8LinearWrapper(lora)
    assert wrap.backend == "native"
    x = torch.randn(3, 37, K, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y = wrap(x)
        y_ref, w_bf, w_f8_ref, w_scale_ref = _ref_native(lora, x)
    w_f8, w_scale = weight_fp8(lora.base_layer.weight_view(), torch.bfloat16)
    assert float(w_scale) == float(w_scale_ref)
    assert torch.equal(w_f8.view(torch.uint8), w_f8_ref.view(torch.uint8))
    assert torch.equal(y, y_ref)
    # grad_x of the base product: grad_y @ w (the frozen weight, activation dtype)
    xg = x.detach().clone().requires_grad_(True)
    gy = torch.randn(3, 37, N, device="cuda", dtype=torch.bfloat16)
    wrap(xg).backward(gy)
    A = lora.lora_A.detach().to(torch.bfloat16)
    B = lora.lora_B.detach().to(torch.bfloat16)
    want = (gy.float() @ w_bf.float() + ((gy @ B).float() * lora.scaling) @ A.float())
    err = (xg.grad.float() - want).abs().max().item()
    assert err <= 2e-2 * want.pow(2).mean().sqrt().item() + 1e-2, err


@pytest.mark.gpu
def test_native_fp8_cache_and_fallbacks():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")
    lora = _gpu_layer(256, 512, 4, True, False, seed=3).eval()
    wrap = FP8LinearWrapper(lora)
    x = torch.randn(16, 512, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        wrap(x)
        first = wrap._cache
        wrap(x)
        assert wrap._cache is first  # the e4m3 weight is kept while the codes are unchanged
        lora.base_layer.weight_quant.add_(0)  # an in-place write bumps the version
        y = wrap(x)
        assert wrap._cache is not first
        assert torch.equal(y, _ref_native(lora, x)[0])
    # out features not a multiple of 16: the wrapped layer runs unchanged
    odd = _gpu_layer(250, 512, 4, False, False, seed=4).eval()
    w_odd = FP8LinearWrapper(odd)
    with torch.no_grad():
        assert torch.equal(w_odd(x), odd(x))
    # fp32 activations: unchanged as well
    with torch.no_grad():
        assert torch.equal(wrap(x.float()), lora(x.float()))
