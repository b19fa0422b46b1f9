"""State dicts interchange with the reference: the buffers of QuantLinear and
LoRALinear keep the reference's names, dtypes and flat layouts
(quant_linear.py:38-45, double_quant.py:185-196 of the reference), so a
checkpoint the reference wrote loads unchanged (tests/golden/state_dicts.npz,
written by the reference itself through tests/golden/make_golden.py).

The CPU test compares the key sets and dtypes; the GPU test loads each
reference state dict into a freshly built layer of this package and checks
its forward output against the reference's.
"""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

GOLD = os.path.join(os.path.dirname(__file__), "golden", "state_dicts.npz")
CASES = ["nf4_bias", "nf4dq", "int8"]


def _load(case):
    z = np.load(GOLD)
    sd = {}
    for k in z.files:
        if k.startswith(f"{case}/sd/"):
            key = k[len(f"{case}/sd/"):]
            dt = getattr(torch, str(z[f"{case}/dtype/{key}"]))
            a = z[k]
            if dt in (torch.bfloat16, torch.float16):
                t = torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(dt)
            elif dt == torch.float8_e4m3fnuz:
                t = torch.from_numpy(a.astype(np.uint8)).view(dt)
            else:
                t = torch.from_numpy(np.ascontiguousarray(a)).to(dt)
            sd[key] = t
    N, K, M, bits, bias, dq = (int(v) for v in z[f"{case}/meta"])
    return sd, (N, K, M, bits, bool(bias), bool(dq)), z[f"{case}/x"], z[f"{case}/y"]


@pytest.mark.parametrize("case", [c for c in CASES if c != "nf4dq"])
def test_state_dict_keys_and_dtypes_match_reference(case):
    """An unquantized layer of this package already has the reference's
    state-dict keys; once quantized buffers are assigned, the dtypes match."""
    from rocm_qlora import LoRALinear, QuantLinear
    sd, (N, K, M, bits, bias, dq), _, _ = _load(case)
    ql = QuantLinear(K, N, bits=bits, bias=bias, block_size=64)
    lora = LoRALinear(ql, r=8, lora_alpha=16)
    ours = lora.state_dict()
    assert set(ours) == set(sd)
    lora.load_state_dict(sd, strict=True)
    for k, v in lora.state_dict().items():
        assert v.shape == sd[k].shape, k
        if not k.endswith("bias"):  # bias is copied into the module's own dtype, as in the reference
            assert v.dtype == sd[k].dtype, k
        assert torch.equal(v.to(sd[k].dtype), sd[k]), k


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_reference_state_dict_loads_and_runs(case):
    from oracle import oracle as orc
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora import _native as nat
    from tests.gpu_util import from_bits, to_f32
    from tests.tolerance import assert_matmul_close
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")
    sd, (N, K, M, bits, bias, dq), xb, yb = _load(case)
    # a layer of the same shape quantized from unrelated weights, then the
    # reference's checkpoint loaded over it
    lin = nn.Linear(K, N, bias=bias, dtype=torch.bfloat16, device="cuda")
    ql = QuantLinear.from_linear(lin, bits=bits)
    if dq:
        ql.enable_double_quant()
    lora = LoRALinear(ql, r=8, lora_alpha=16).cuda().eval()
    lora.load_state_dict({k: v.cuda() for k, v in sd.items()}, strict=True)
    x = from_bits(xb, 1).reshape(M, K).cuda()
    with torch.no_grad():
        y = lora(x)
    assert_matmul_close(to_f32(y), orc.to_f32(yb, 1).reshape(M, N), 1, label=f"reference state dict {case}")
