"""GPU parity of the quantize / dequantize kernels (bit-exact).

Each case runs the sm_100a kernels through the package API (which calls the
C ABI) and compares codes, scales, second-level scales and dequantized values
bit for bit with the reference's own outputs (tests/golden) and with the C
oracle on larger seeded inputs.
"""
import hashlib
import os
import unittest.mock as mock

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.gpu_util import from_bits, same_float_bits, to_bits

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def cases(z, suffix):
    return sorted({k.rsplit("/", 1)[0] for k in z.files if k.endswith("/" + suffix)})


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable: " + ("no CUDA device" if not torch.cuda.is_available()
                                                    else "library missing or device is not sm_100"))


@pytest.mark.parametrize("case", cases(load("nf4.npz"), "packed"))
def test_nf4_quantize_golden(case):
    from rocm_qlora.quantization import quantize_int4, dequantize_int4
    z = load("nf4.npz")
    dt, bs = int(z[f"{case}/dtype"]), int(z[f"{case}/bs"])
    x = from_bits(z[f"{case}/x"], dt).cuda()
    p, s = quantize_int4(x, block_size=bs)
    assert p.is_cuda and p.dtype == torch.uint8
    assert np.array_equal(to_bits(p), z[f"{case}/packed"])
    assert same_float_bits(to_bits(s), z[f"{case}/scales"], dt)
    d = dequantize_int4(p, s, block_size=bs)
    assert d.dtype == torch.float32
    assert same_float_bits(to_bits(d), z[f"{case}/deq"], 0)


@pytest.mark.parametrize("case", cases(load("int8.npz"), "q"))
def test_int8_quantize_golden(case):
    from rocm_qlora.quantization import quantize_int8, dequantize_int8
    z = load("int8.npz")
    dt = int(z[f"{case}/dtype"])
    x = from_bits(z[f"{case}/x"], dt).cuda()
    if case.startswith("rows"):
        q, s = quantize_int8(x, per_channel=True)
        d = dequantize_int8(q, s)
    else:
        bs = int(z[f"{case}/bs"])
        q, s = quantize_int8(x, block_size=bs)
        d = dequantize_int8(q, s, block_size=bs)
    assert np.array_equal(to_bits(q).reshape(-1), z[f"{case}/q"].reshape(-1))
    assert same_float_bits(to_bits(s), z[f"{case}/scales"], dt)
    if f"{case}/deq" in z.files:
        assert same_float_bits(to_bits(d), z[f"{case}/deq"], 0)


@pytest.mark.parametrize("case", cases(load("double_quant.npz"), "c2"))
def test_double_quant_golden(case):
    import torch.nn as nn
    from rocm_qlora.quantization import QuantLinear, double_quantize, double_dequantize
    from rocm_qlora.quantization.double_quant import DoubleQuantState
    z = load("double_quant.npz")
    if case.startswith("api"):
        dt = int(z[f"{case}/dtype"])
        N, K = (int(v) for v in z[f"{case}/shape"])
        w = from_bits(z[f"{case}/w"], dt).reshape(N, K).cuda()
        lin = nn.Linear(K, N, bias=False, device="cuda", dtype=w.dtype)
        with torch.no_grad():
            lin.weight.copy_(w)
        ql = QuantLinear.from_linear(lin, bits=4)
        assert np.array_equal(to_bits(ql.weight_quant), z[f"{case}/packed"])
        assert same_float_bits(to_bits(ql.weight_scales), z[f"{case}/scales"], dt)
        assert ql.enable_double_quant()
        c2, c2s, packed = ql.c2, ql.c2_scales, ql.weight_quant
        assert ql.weight_scales.numel() == 0 and ql.c2.dtype == torch.float8_e4m3fnuz
        deq = ql.dequantized_weight()
    else:
        fp8 = case.endswith("1")
        w = torch.from_numpy(z[f"{case}/w"]).cuda()
        if fp8:
            st = double_quantize(w)
        else:
            with mock.patch("rocm_qlora.quantization.double_quant._has_fp8", return_value=False):
                st = double_quantize(w)
            assert st.c2.dtype == torch.int8 and st.use_fp8_c2 is False
        c2, c2s, packed = st.c2, st.c2_scales, st.W_quant
        deq = double_dequantize(st)
    assert np.array_equal(to_bits(packed), z[f"{case}/packed"])
    assert np.array_equal(to_bits(c2).view(np.uint8).reshape(-1), z[f"{case}/c2"].view(np.uint8).reshape(-1))
    assert np.array_equal(to_bits(c2s).reshape(-1).view(np.uint32), z[f"{case}/c2_scales"].view(np.uint32))
    assert same_float_bits(to_bits(deq), z[f"{case}/deq"], 0)


def test_config1_codes_scales_hash():
    """Config 1 (W 4096x4096 fp32 N(0,0.02), seed 0): GPU codes and scales
    hash to the reference's."""
    from rocm_qlora.quantization import quantize_int4
    from tests.inputs import config1
    z = load("config1.npz")
    c1 = config1()
    p, s = quantize_int4(c1.W.cuda().flatten(), block_size=64)
    assert hashlib.sha256(to_bits(p).tobytes()).hexdigest() == str(z["codes_sha256"])
    assert hashlib.sha256(to_bits(s).tobytes()).hexdigest() == str(z["scales_sha256"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_nf4_large_vs_oracle(dtype):
    """A 2048x4096 weight (plus a ragged tail) against the C oracle."""
    from rocm_qlora.quantization import quantize_int4, dequantize_int4
    from rocm_qlora.kernels import dequantize_nf4_triton
    g = torch.Generator().manual_seed(11)
    w = (torch.randn(2048 * 4096 + 37, generator=g) * 0.02).to(dtype)
    dt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]
    p, s = quantize_int4(w.cuda())
    rp, rs = orc.nf4_quantize(to_bits(w), dt, 64)
    assert np.array_equal(to_bits(p), rp)
    assert np.array_equal(to_bits(s).view(np.uint8), rs.view(np.uint8))
    d = dequantize_int4(p, s)
    rd = orc.nf4_dequantize(rp, rs, dt)
    assert np.array_equal(to_bits(d).view(np.uint32), rd.view(np.uint32))
    db = dequantize_nf4_triton(p, s)
    assert db.dtype == torch.bfloat16
    assert np.array_equal(to_bits(db), orc.f32_to_bf16_bits(rd))


def test_dq_large_vs_oracle():
    """Double quant of a 4096x4096 bf16 weight via enable_double_quant: c2
    groups of 256 blocks straddle rows when K/64 is not a multiple of 256."""
    import torch.nn as nn
    from rocm_qlora.quantization import QuantLinear
    g = torch.Generator().manual_seed(12)
    for N, K in ((512, 4096), (300, 64 * 300)):
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device="cuda")
        with torch.no_grad():
            lin.weight.copy_(w.cuda())
        ql = QuantLinear.from_linear(lin, bits=4)
        ql.enable_double_quant()
        rp, rs = orc.nf4_quantize(to_bits(w), 1, 64)
        rc2, rc2s = orc.enable_double_quant(rp, rs, 1, N * K)
        assert np.array_equal(to_bits(ql.weight_quant), rp)
        assert np.array_equal(to_bits(ql.c2).reshape(-1), rc2)
        assert np.array_equal(to_bits(ql.c2_scales).reshape(-1).view(np.uint32), rc2s.view(np.uint32))


def test_device_agnostic_cpu_inputs():
    """CPU tensors in, CPU tensors out (computed on the GPU), as the
    reference's test_device_agnostic expects."""
    from rocm_qlora.quantization import quantize_int8, dequantize_int8, quantize_int4, dequantize_int4
    t = torch.randn(128)
    q8, s8 = quantize_int8(t)
    q4, s4 = quantize_int4(t)
    assert q8.device.type == "cpu" and dequantize_int8(q8, s8).device.type == "cpu"
    assert q4.device.type == "cpu" and dequantize_int4(q4, s4).device.type == "cpu"
    rp, rs = orc.nf4_quantize(t.numpy(), 0, 64)
    assert np.array_equal(q4.numpy(), rp)


def test_roundtrip_error_bounds():
    """The reference's tolerance tests (tests/test_quant_ops.py:13-63)."""
    from rocm_qlora.quantization import quantize_int8, dequantize_int8, quantize_int4, dequantize_int4
    torch.manual_seed(42)
    for bs in (64, 128):
        x = torch.randn(1024, device="cuda") * 2.0
        x[0] = 100.0
        q, s = quantize_int8(x, block_size=bs)
        d = dequantize_int8(q, s, block_size=bs)
        assert (x - d[:x.numel()]).abs().max() < 0.01 * x.abs().max()
        x = torch.randn(1024, device="cuda")
        p, s = quantize_int4(x, block_size=bs)
        d = dequantize_int4(p, s, block_size=bs)
        assert (x - d[:x.numel()]).abs().max() < 0.15 * x.abs().max()
        assert p.numel() * 2 >= x.numel()


def test_empty_and_tiny_inputs():
    from rocm_qlora.quantization import quantize_int4, quantize_int8
    p, s = quantize_int4(torch.zeros(0, device="cuda"))
    assert p.numel() == 0
    p, s = quantize_int4(torch.tensor([0.5, -0.25, 0.125], device="cuda"))
    rp, rs = orc.nf4_quantize(np.array([0.5, -0.25, 0.125], np.float32), 0, 64)
    assert np.array_equal(p.cpu().numpy(), rp)
    x = torch.tensor([3.0], dtype=torch.bfloat16)
    q, s = quantize_int8(x.cuda())
    rq, rs = orc.int8_quantize(to_bits(x), 1, 64)
    assert q.numel() == 64 and np.array_equal(q.cpu().numpy(), rq)  # bf16(3/127) makes 3.0 -> 126
