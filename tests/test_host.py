"""CPU-only tests of the host side: the C-ABI library loads and exports every
symbol include/rq_b200.h declares, the Python API mirrors the reference's
surface and validation, and nothing computes without the GPU kernels."""
import ctypes
import os
import re
import subprocess

import pytest
import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rq_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"RQ_API\s+[\w\s\*]+?\b((?:rq|launch)_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from rocm_qlora import _native as nat
    L = nat.load_library()
    syms = header_symbols()
    assert len(syms) >= 16
    for s in syms:
        assert hasattr(L, s), f"{s} missing from {nat.LIB_PATH}"
    assert set(syms) == set(nat.exported_symbols())
    out = subprocess.run(["nm", "-D", "--defined-only", nat.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T ((?:rq|launch)_\w+)", out))
    assert exported == set(syms)


def test_library_is_sm100a():
    """The shared library carries sm_100a device code (checked from the
    build log's target list, not by decoding the binary)."""
    from rocm_qlora import _native as nat
    L = nat.load_library()
    assert L.rq_abi_version() == 3
    mk = open(os.path.join(ROOT, "rocm-qlora_b200", "Makefile")).read()
    assert "arch=compute_100a,code=sm_100a" in mk


def test_status_strings():
    from rocm_qlora import _native as nat
    L = nat.load_library()
    assert L.rq_status_string(0) == b"ok"
    assert b"workspace" in L.rq_status_string(-5)
    assert b"sm_100" in L.rq_status_string(-6)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    """Without a CUDA device every compute call raises instead of computing
    on the CPU."""
    from rocm_qlora import _native as nat
    from rocm_qlora.quantization import quantize_int4, dequantize_int8
    with pytest.raises(nat.NativeUnavailable):
        quantize_int4(torch.randn(64))
    with pytest.raises(nat.NativeUnavailable):
        dequantize_int8(torch.zeros(64, dtype=torch.int8), torch.ones(1))
    from rocm_qlora import QuantLinear
    with pytest.raises(nat.NativeUnavailable):
        QuantLinear.from_linear(nn.Linear(64, 64), bits=4)


def test_config_validation_and_roundtrip():
    from rocm_qlora import RocmQLoraConfig
    c = RocmQLoraConfig(bits=4, lora_r=16)
    assert c.to_dict()["bits"] == 4 and c.target_modules == ["q_proj", "v_proj", "k_proj", "o_proj"]
    assert RocmQLoraConfig.from_dict(c.to_dict()).to_dict() == c.to_dict()
    with pytest.raises(ValueError, match="only supports 4 or 8 bits"):
        RocmQLoraConfig(bits=3)


def test_quantize_model_rejects_bits():
    from rocm_qlora import quantize_model
    with pytest.raises(ValueError, match="Only 4 and 8 bits are supported"):
        quantize_model(nn.Linear(128, 128), bits=3)


def test_quantlinear_constructor_buffers():
    from rocm_qlora import QuantLinear
    ql = QuantLinear(64, 128, bits=4)
    names = set(dict(ql.named_buffers()))
    assert {"weight_quant", "weight_scales", "weight_zeros", "bias"} <= names
    assert ql.weight_quant.dtype == torch.uint8
    assert QuantLinear(64, 128, bits=8).weight_quant.dtype == torch.int8
    assert sum(p.numel() for p in ql.parameters()) == 0
    assert "in=64, out=128, bits=4" in repr(ql)


def test_lora_layer_params_without_compute():
    from rocm_qlora import LoRALinear, QuantLinear
    lora = LoRALinear(QuantLinear(64, 128, bits=8), r=8)
    trainable = [n for n, p in lora.named_parameters() if p.requires_grad]
    assert trainable == ["lora_A", "lora_B"]
    assert lora.get_trainable_params() == 1536
    assert torch.count_nonzero(lora.lora_B) == 0
    assert lora.scaling == 2.0


def test_double_quant_savings_estimate():
    from rocm_qlora.quantization import estimate_double_quant_savings
    s = estimate_double_quant_savings(torch.empty(4096, 4096))
    assert 0.35 < s["bits_saved_per_param"] < 0.40
    assert s["saved_bytes"] > 0


def test_double_quant_state_defaults():
    from rocm_qlora.quantization import DoubleQuantState
    st = DoubleQuantState(W_quant=torch.zeros(1, dtype=torch.uint8), c2=torch.zeros(1), c2_scales=torch.zeros(1),
                          original_shape=(10, 10))
    assert st.blocksize_1 == 64 and st.blocksize_2 == 256


def test_public_names_match_reference_surface():
    import rocm_qlora
    import rocm_qlora.kernels as k
    import rocm_qlora.quantization as q
    for name in ["quantize_model", "QuantLinear", "LoRALinear", "enable_all_kernels", "RocmQLoraConfig",
                 "fused_dequant_int8_matmul", "fused_dequant_nf4_matmul", "get_device_info", "is_triton_available"]:
        assert hasattr(rocm_qlora, name)
    for name in ["quantize_int8", "dequantize_int8", "quantize_int4", "dequantize_int4", "QuantLinear",
                 "double_quantize", "double_dequantize", "DoubleQuantState", "estimate_double_quant_savings",
                 "patch_quant_linear_for_double_quant"]:
        assert hasattr(q, name)
    for name in ["get_kernel_config", "get_device_info", "is_triton_available", "fused_dequant_int8_matmul",
                 "fused_dequant_nf4_matmul", "dequantize_nf4_triton"]:
        assert hasattr(k, name)
    info = k.get_device_info()
    assert {"arch", "compute_units", "vram_gb", "wavefront_size", "triton_available"} <= set(info)


def test_workspace_size_query():
    from rocm_qlora import _native as nat
    L = nat.load_library()
    assert L.rq_linear_workspace_bytes(16, 4096, 4096, 0) == 256
    assert L.rq_linear_workspace_bytes(16, 4096, 4096, 16) > 256
    assert L.rq_linear_workspace_bytes(-1, 1, 1, 1) == -1


def test_weight_view_cache_follows_buffers():
    """QuantLinear.weight_view() is reused while the quantized buffers are
    unchanged and rebuilt after an in-place write, a replaced buffer or a
    format change; inference tensors are never cached."""
    import torch
    from rocm_qlora import QuantLinear
    ql = QuantLinear(256, 128, bits=4)
    ql.weight_quant = torch.zeros(128 * 256 // 2, dtype=torch.uint8)
    ql.weight_scales = torch.ones(128 * 256 // 64)
    w1 = ql.weight_view()
    assert ql.weight_view() is w1
    assert w1.args() is w1.args()
    ql.weight_quant.bitwise_or_(0)  # in place: the version counter moves
    w2 = ql.weight_view()
    assert w2 is not w1 and ql.weight_view() is w2
    ql.weight_scales = ql.weight_scales.clone()  # a new tensor
    w3 = ql.weight_view()
    assert w3 is not w2 and w3.scales.data_ptr() == ql.weight_scales.data_ptr()
    ql.block_size = 32
    assert ql.weight_view() is not w3
    with torch.inference_mode():
        qi = QuantLinear(256, 128, bits=4)
    assert qi.weight_view() is not qi.weight_view()


def test_export_helpers_host_side():
    """The export module's host-only helpers (size estimate, conversion
    steps) -- the reference's gguf_export.py API."""
    from rocm_qlora.export import estimate_gguf_size, get_gguf_conversion_instructions
    e = estimate_gguf_size(7_000_000_000, "q4_k_m")
    assert e["bits_per_param"] == 4.5 and e["quant_type"] == "q4_k_m"
    assert abs(e["estimated_size_gb"] - 7e9 * 4.5 / 8 / 1e9 * 1.05) < 0.01
    assert estimate_gguf_size(10, "nope")["bits_per_param"] == 4.5
    text = get_gguf_conversion_instructions("/tmp/m.safetensors")
    assert "convert_hf_to_gguf.py /tmp/m.safetensors" in text and "q4_k_m" in text


def test_cast_param_cache():
    """Adapter casts are reused while the parameter is unchanged and redone
    after an in-place update or forget_casts()."""
    from rocm_qlora.quantization import layer_ops as lo
    p = torch.nn.Parameter(torch.randn(4, 8))
    a = lo.cast_param(p, torch.bfloat16)
    assert lo.cast_param(p, torch.bfloat16) is a
    with torch.no_grad():
        p.add_(1)
    c = lo.cast_param(p, torch.bfloat16)
    assert c is not a and torch.equal(c, p.detach().bfloat16())
    p.data.zero_()  # not seen by the version counter ...
    lo.forget_casts(p)  # ... hence the explicit reset
    assert float(lo.cast_param(p, torch.bfloat16).abs().sum()) == 0


def test_torch_extension_registers_the_layer_ops():
    """The thin torch extension over the C ABI (librq_torch_ops.so) loads
    without a GPU and registers both layer operators; their Meta kernels
    give the output shapes (tracing)."""
    import torch
    from rocm_qlora import _native as nat
    assert nat.ops(), "librq_torch_ops.so missing or not loadable"
    ops = torch.ops.rocm_qlora
    x = torch.empty(5, 128, device="meta", dtype=torch.bfloat16)
    q = torch.empty(32 * 128 // 2, device="meta", dtype=torch.uint8)
    ws = torch.empty(256, device="meta", dtype=torch.uint8)
    y = ops.linear_forward(x, 0, q, None, None, None, 32, 128, 64, None, None, None, None, 1.0, ws)
    assert y.shape == (5, 32) and y.dtype == torch.bfloat16
    dy = torch.empty(5, 32, device="meta", dtype=torch.float16)
    dx = ops.linear_dx(dy, 0, q, None, None, None, 32, 128, 64, None, None, 1.0, ws)
    assert dx.shape == (5, 128) and dx.dtype == torch.float16
