"""Merged weights on the GPU (rq_merge_lora): LoRALinear.merge_lora and the
fp16 export path (_export_dequant_layer, merge_and_export_fp16), against
the oracle restating the reference's two rounding sequences:

  merge_lora (lora_layer.py:72-113):  fp16(deq(W) + (B @ A) * s), fp32 sums
  export (gguf_export.py:30-80):      fp16(deq(W)) + fp16((B @ A) * s)

The delta's fp32 dot product may sum in another order than the oracle's,
so a result may sit one fp16 ulp away where the fp32 sum lies next to a
rounding boundary (for the export, one ulp of the rounded delta, which is
the larger where weight and delta cancel); at least 99 % must match bit for
bit.
"""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import oracle as orc
from tests.test_gpu_linear import build_layer, oracle_wdeq

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _ref_delta(A, B, s):
    return (B.astype(np.float64) @ A.astype(np.float64)).astype(np.float32) * np.float32(s)


def _ulp16(a):
    return np.abs(np.spacing(np.asarray(a, np.float32).astype(np.float16)).astype(np.float32))


def _check(got, want, delta=None):
    """One fp16 ulp of the result; with `delta` (the export's rounding, the
    delta rounded on its own) also one ulp of fp16(delta): where the weight
    and the delta cancel, the sum of the two fp16 values is exact and a
    one-ulp flip of fp16(delta) passes through unchanged."""
    got = got.detach().float().cpu().numpy()
    diff = np.abs(got - want)
    ulp = _ulp16(want)
    if delta is not None:
        ulp = np.maximum(ulp, _ulp16(delta))
    assert np.all(diff <= ulp), f"max diff {diff.max()} beyond one fp16 ulp"
    exact = float(np.mean(diff == 0))
    assert exact >= 0.99, f"only {exact:.4f} of the merged weights are bit-identical"
    return exact


def _layer(fmt, N, K, r, seed):
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.quantization import quantize_int8
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    A = (torch.rand(r, K, generator=g) * 2 - 1) / K ** 0.5
    B = torch.randn(N, r, generator=g) * 0.01
    if fmt == "int8_row":
        ql = QuantLinear(K, N, bits=8, bias=False).cuda()
        q, s = quantize_int8(W.cuda(), per_channel=True)
        ql.weight_quant, ql.weight_scales = q, s
        lora = LoRALinear(ql, r=r, lora_alpha=2 * r).cuda()
        with torch.no_grad():
            lora.lora_A.copy_(A.cuda())
            lora.lora_B.copy_(B.cuda())
        return lora
    return build_layer(W, 8 if fmt == "int8" else 4, fmt == "nf4_dq", None, r, 2 * r, A, B)


def _wdeq(lora):
    from tests.gpu_util import to_bits
    ql = lora.base_layer
    N, K = ql.out_features, ql.in_features
    if ql.bits == 8 and ql.weight_quant.dim() == 2:
        return orc.int8_dequantize(to_bits(ql.weight_quant).reshape(-1), to_bits(ql.weight_scales), orc.BF16,
                                   rows=N, cols=K).reshape(N, K)
    return oracle_wdeq(ql, N, K)


@pytest.mark.parametrize("fmt,N,K,r", [("nf4_dq", 1024, 4096, 16), ("nf4", 600, 1088, 8), ("int8", 520, 1024, 64),
                                       ("int8_row", 256, 2048, 100), ("nf4_dq", 4096, 11008, 16)])
def test_merge_lora_matches_reference_rounding(fmt, N, K, r):
    from rocm_qlora.export.gguf_export import _export_dequant_layer
    lora = _layer(fmt, N, K, r, seed=N + r)
    A = lora.lora_A.detach().cpu().numpy()
    B = lora.lora_B.detach().cpu().numpy()
    w = _wdeq(lora)
    delta = _ref_delta(A, B, lora.scaling)
    exported = _export_dequant_layer(lora)          # fp16(W) + fp16(delta), in fp16
    assert exported.dtype == torch.float16 and exported.shape == (N, K)
    _check(exported, _f16(_f16(w) + _f16(delta)), delta)
    x = torch.randn(3, K, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        y_before = lora(x)
    lora.merge_lora()                               # fp16(W + delta), fp32 sum
    merged = lora.base_layer.merged_fp16_weight
    _check(merged, _f16(w + delta))
    assert float(lora.lora_A.abs().sum()) == 0 and float(lora.lora_B.abs().sum()) == 0
    with torch.no_grad():
        y_after = lora(x)
    assert torch.allclose(y_after.float(), y_before.float(), atol=5e-2, rtol=5e-2)
    lora.unmerge_lora()
    assert not lora.base_layer.merged_mode


def test_merge_and_export_fp16_writes_hf_layout(tmp_path):
    from safetensors.torch import load_file
    from rocm_qlora import LoRALinear, quantize_model
    from rocm_qlora.export import merge_and_export_fp16
    from rocm_qlora.export.gguf_export import _export_dequant_layer

    class Tiny(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(256, 256)
            self.v_proj = nn.Linear(256, 512, bias=False)
            self.norm = nn.LayerNorm(256)

    torch.manual_seed(0)
    model = quantize_model(Tiny().cuda(), bits=4, lora_r=8, lora_alpha=16, target_modules=["q_proj", "v_proj"])
    model.cuda()
    with torch.no_grad():
        model.q_proj.lora_B.normal_(0, 0.01)
    path = os.path.join(tmp_path, "merged.safetensors")
    assert merge_and_export_fp16(model, path, model_config={"model_type": "tiny"}) == path
    sd = load_file(path)
    assert set(sd) == {"q_proj.weight", "q_proj.bias", "v_proj.weight", "norm.weight", "norm.bias"}
    assert all(t.dtype == torch.float16 for t in sd.values())
    assert sd["v_proj.weight"].shape == (512, 256)
    assert torch.equal(sd["q_proj.weight"], _export_dequant_layer(model.q_proj).cpu())
    assert os.path.exists(os.path.join(tmp_path, "config.json"))
