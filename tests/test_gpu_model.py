"""Model-level orchestration on the GPU: quantize_model + enable_all_kernels
on a small transformer-shaped module tree, then forward and backward
through the swapped layers (the behaviour the reference checks in
tests/test_quantize_model.py:56-81, here on the B200 kernels).

Each swapped layer's output is also checked against the oracle of the
reference's eager path (dequantize + F.linear + the adapter, with the
reference's per-op roundings), fed with the GPU's own input to that layer,
so the check is per layer and does not compound along the chain.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import oracle as orc
from tests.gpu_util import to_f32
from tests.test_gpu_linear import DTC, oracle_wdeq
from tests.tolerance import assert_matmul_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")


class Block(nn.Module):
    """Attention-shaped projections and an MLP: SwiGLU (gate/up/down, as in
    Llama; the down projection sees centred activations) or ReLU (the down
    projection sees activations that all share a sign)."""

    def __init__(self, d, f, relu):
        super().__init__()
        self.relu = relu
        self.q_proj = nn.Linear(d, d, bias=False)
        self.k_proj = nn.Linear(d, d, bias=False)
        self.v_proj = nn.Linear(d, d, bias=True)
        self.o_proj = nn.Linear(d, d, bias=False)
        self.gate_proj = nn.Linear(d, f, bias=False)
        self.up_proj = nn.Linear(d, f, bias=False)
        self.down_proj = nn.Linear(f, d, bias=False)
        self.norm = nn.LayerNorm(d)

    def forward(self, x):
        h = self.o_proj(self.q_proj(x) + self.k_proj(x) + self.v_proj(x))
        x = self.norm(x + h)
        a = torch.relu(self.up_proj(x)) if self.relu else nn.functional.silu(self.gate_proj(x)) * self.up_proj(x)
        return x + self.down_proj(a)


class TinyModel(nn.Module):
    def __init__(self, d=256, f=512, n=3, relu=False):
        super().__init__()
        self.blocks = nn.ModuleList([Block(d, f, relu) for _ in range(n)])
        self.tiny = nn.Linear(32, 32)   # below quantize_model's 64-feature floor
        self.head = nn.Linear(d, 64)    # not a target

    def forward(self, x):
        for b in self.blocks:
            x = b(x)
        return self.head(x)


TARGETS = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


@pytest.fixture
def decode_mode():
    """Sets the decode GEMV numerics for one test and restores the default."""
    from rocm_qlora import _native as nat
    yield nat.set_decode_exact
    nat.set_decode_exact(False)


def _taps(model):
    """Inputs and outputs of every LoRALinear in the model (forward hooks)."""
    from rocm_qlora import LoRALinear
    seen = []
    hooks = [m.register_forward_hook(lambda mod, inp, out: seen.append((mod, inp[0].detach(), out.detach())))
             for m in model.modules() if isinstance(m, LoRALinear)]
    return seen, hooks


# (bits, dtype, ReLU MLP, exact decode numerics): the ReLU model runs the
# decode GEMV with the exact numerics (the reference's own weights), meant
# for activations that share a sign; the SwiGLU model runs the default
CASES = [(4, torch.bfloat16, False, False), (8, torch.bfloat16, False, False), (4, torch.float32, False, False),
         (8, torch.float32, False, False), (4, torch.bfloat16, True, True), (4, torch.float16, True, True)]


@pytest.mark.parametrize("bits,dt,relu,exact", CASES)
def test_quantize_model_forward_backward(bits, dt, relu, exact, decode_mode):
    from rocm_qlora import LoRALinear, QuantLinear, enable_all_kernels, quantize_model
    decode_mode(exact)
    torch.manual_seed(bits)
    model = TinyModel(relu=relu).to(device="cuda", dtype=dt)
    targets = [t for t in TARGETS if not (relu and t == "gate_proj")]
    model = quantize_model(model, bits=bits, lora_r=8, lora_alpha=16, lora_dropout=0.05, target_modules=targets)
    n_swapped = sum(isinstance(m, LoRALinear) for m in model.modules())
    assert n_swapped == 3 * len(targets)
    assert isinstance(model.tiny, nn.Linear) and isinstance(model.head, nn.Linear)
    # like the reference's, the walk meets every QuantLinear twice: as the
    # LoRALinear's base_layer and as a module of its own
    assert enable_all_kernels(model) == 2 * n_swapped
    assert all(m.use_triton_kernel for m in model.modules() if isinstance(m, QuantLinear))
    model.to("cuda")
    with torch.no_grad():  # adapters away from their zero init, so the adapter term is checked too
        for m in model.modules():
            if isinstance(m, LoRALinear):
                m.lora_B.normal_(0.0, 0.02)

    # eval: every swapped layer against the oracle on the layer's own input
    model.eval()
    seen, hooks = _taps(model)
    x = torch.randn(12, 256, device="cuda", dtype=dt)
    with torch.no_grad():
        out = model(x)
    for h in hooks:
        h.remove()
    assert out.shape == (12, 64) and torch.isfinite(out.float()).all()
    assert len(seen) == n_swapped
    xdt = DTC[dt]
    for mod, xin, yout in seen:
        ql = mod.base_layer
        wdeq = oracle_wdeq(ql, ql.out_features, ql.in_features)
        bias = ql.bias.float().cpu().numpy() if ql.bias is not None else None
        y_ref = orc.loralinear_forward(to_f32(xin), wdeq, bias, mod.lora_A.detach().float().cpu().numpy(),
                                       mod.lora_B.detach().float().cpu().numpy(), mod.scaling, xdt)
        assert_matmul_close(to_f32(yout), y_ref, xdt)

    # train: LoRA dropout active, gradients reach exactly the trainable parameters
    model.train()
    xg = torch.randn(12, 256, device="cuda", dtype=dt, requires_grad=True)
    model(xg).float().pow(2).mean().backward()
    assert xg.grad is not None and torch.isfinite(xg.grad.float()).all()
    for name, p in model.named_parameters():
        if "lora_A" in name or "lora_B" in name:
            assert p.grad is not None and torch.isfinite(p.grad).all(), name
            assert p.grad.abs().sum() > 0, name
        else:
            assert not p.requires_grad and p.grad is None, name
