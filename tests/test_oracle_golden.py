"""The C/numpy oracle against the reference's own outputs (golden fixtures).

Every fixture in tests/golden/ was produced by the reference package itself
(tests/golden/make_golden.py).  Codes, scales, fp8 second-level scales and
dequantized values must match bit for bit; matmul outputs within the
tolerance used by the GPU parity tests (see tests/tolerance.py).
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import oracle as orc
from tests.tolerance import assert_matmul_close

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def same_bits(a, b, dtype):
    """Bitwise equality of float arrays given as bit patterns, except that any
    NaN equals any NaN (the reference's NaN payloads depend on torch's
    vectorisation and are not part of the format)."""
    fa, fb = orc.to_f32(a.reshape(-1), dtype), orc.to_f32(b.reshape(-1), dtype)
    na, nb_ = np.isnan(fa), np.isnan(fb)
    if not np.array_equal(na, nb_):
        return False
    return np.array_equal(fa[~na].view(np.uint32), fb[~nb_].view(np.uint32))


def cases(z, suffix):
    return sorted({k.rsplit("/", 1)[0] for k in z.files if k.endswith("/" + suffix)})


def test_nf4_table_bits():
    z = load("nf4.npz")
    assert np.array_equal(orc.nf4_table().view(np.uint32), z["table"].view(np.uint32))


@pytest.mark.parametrize("case", cases(load("nf4.npz"), "packed"))
def test_nf4_quantize_matches_reference(case):
    z = load("nf4.npz")
    x, dt, bs = z[f"{case}/x"], int(z[f"{case}/dtype"]), int(z[f"{case}/bs"])
    packed, scales = orc.nf4_quantize(x, dt, bs)
    assert np.array_equal(packed, z[f"{case}/packed"])
    assert same_bits(scales, z[f"{case}/scales"], dt)
    deq = orc.nf4_dequantize(packed, scales, dt, bs)
    assert same_bits(deq, z[f"{case}/deq"], orc.F32)


@pytest.mark.parametrize("case", cases(load("int8.npz"), "q"))
def test_int8_quantize_matches_reference(case):
    z = load("int8.npz")
    x, dt = z[f"{case}/x"], int(z[f"{case}/dtype"])
    if case.startswith("rows"):
        q, s = orc.int8_quantize_rows(x, dt)
        deq = orc.int8_dequantize(q, s, dt, rows=x.shape[0], cols=x.shape[1])
    else:
        bs = int(z[f"{case}/bs"])
        q, s = orc.int8_quantize(x, dt, bs)
        deq = orc.int8_dequantize(q, s, dt, bs)
    assert np.array_equal(q.reshape(-1), z[f"{case}/q"].reshape(-1))
    assert same_bits(s, z[f"{case}/scales"], dt)
    if f"{case}/deq" in z.files:
        assert same_bits(deq, z[f"{case}/deq"], orc.F32)


def test_int8_wrap_case_present():
    """The fixture holds blocks where the reference's int8 cast wraps 128 -> -128."""
    z = load("int8.npz")
    assert (z["wrap/q"] == -128).any()


def test_fp8_e4m3fnuz_codec():
    z = load("double_quant.npz")
    dec = np.array([orc.lib().orc_e4m3fnuz_to_f32(i) for i in range(256)], np.float32)
    ref = z["fp8/decode"]
    assert np.array_equal(np.isnan(dec), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(dec[ok].view(np.uint32), ref[ok].view(np.uint32))
    enc = np.array([orc.lib().orc_f32_to_e4m3fnuz(float(v)) for v in z["fp8/sweep"]], np.uint8)
    assert np.array_equal(enc, z["fp8/encode"])


@pytest.mark.parametrize("case", cases(load("double_quant.npz"), "c2"))
def test_double_quant_matches_reference(case):
    z = load("double_quant.npz")
    if case.startswith("api"):
        dt = int(z[f"{case}/dtype"])
        N, K = (int(v) for v in z[f"{case}/shape"])
        packed, scales = orc.nf4_quantize(z[f"{case}/w"], dt, 64)
        assert np.array_equal(packed, z[f"{case}/packed"])
        assert np.array_equal(scales.view(np.uint8), z[f"{case}/scales"].view(np.uint8))
        c2, c2s = orc.enable_double_quant(packed, scales, dt, N * K)
        fp8 = True
    else:
        fp8 = case.endswith("1")
        w = z[f"{case}/w"]
        packed, c1 = orc.nf4_quantize(w, orc.F32, 64)
        assert np.array_equal(packed, z[f"{case}/packed"])
        c2, c2s = orc.dq_second_level(c1, 256, fp8)
        N, K = w.shape
    assert np.array_equal(c2, z[f"{case}/c2"].view(np.uint8))
    assert np.array_equal(c2s.view(np.uint32), z[f"{case}/c2_scales"].view(np.uint32))
    deq = orc.double_dequantize(packed, c2, c2s, N * K, 64, fp8)
    ref = z[f"{case}/deq"].reshape(-1)
    assert np.array_equal(deq.view(np.uint32), ref.view(np.uint32))


def _layer_case(z, name):
    N, K, M, wdt, xdt, bits, bias, dq, r, alpha = (int(v) for v in z[f"{name}/meta"])
    return dict(N=N, K=K, M=M, wdt=wdt, xdt=xdt, bits=bits, bias=bias, dq=dq, r=r, alpha=alpha)


@pytest.mark.parametrize("name", cases(load("layers.npz"), "y"))
def test_layer_oracle_matches_reference(name):
    z = load("layers.npz")
    c = _layer_case(z, name)
    N, K, M, xdt = c["N"], c["K"], c["M"], c["xdt"]
    w = z[f"{name}/w"]
    if c["bits"] == 4:
        packed, scales = orc.nf4_quantize(w, c["wdt"], 64)
        assert np.array_equal(packed, z[f"{name}/qweight"])
        if c["dq"]:
            c2, c2s = orc.enable_double_quant(packed, scales, c["wdt"], N * K)
            assert np.array_equal(c2, z[f"{name}/c2"].view(np.uint8))
            wdeq = orc.double_dequantize(packed, c2, c2s, N * K)
        else:
            wdeq = orc.nf4_dequantize(packed, scales, c["wdt"])[: N * K]
    else:
        q, scales = orc.int8_quantize(w, c["wdt"], 64)
        assert np.array_equal(q, z[f"{name}/qweight"])
        wdeq = orc.int8_dequantize(q, scales, c["wdt"], 64)[: N * K]
    wdeq = wdeq.reshape(N, K)
    x = orc.to_f32(z[f"{name}/x"], xdt).reshape(M, K)
    dy = orc.to_f32(z[f"{name}/dy"], xdt).reshape(M, N)
    A = z[f"{name}/A"].reshape(c["r"], K)
    B = z[f"{name}/B"].reshape(N, c["r"])
    bias = orc.to_f32(z[f"{name}/bias"], c["wdt"]) if c["bias"] else None
    s = c["alpha"] / c["r"]
    y = orc.loralinear_forward(x, wdeq, bias, A, B, s, xdt)
    dx = orc.loralinear_dx(dy, wdeq, A, B, s, xdt)
    assert_matmul_close(y, orc.to_f32(z[f"{name}/y"], xdt).reshape(M, N), xdt)
    assert_matmul_close(dx, orc.to_f32(z[f"{name}/dx"], xdt).reshape(M, K), xdt)


def test_config1_codes_and_scales_pinned():
    """Config 1 (W 4096x4096 fp32 seed 0): the oracle's codes and scales hash
    to the reference's."""
    from tests.inputs import config1
    z = load("config1.npz")
    c1 = config1()
    w = c1.W.numpy().reshape(-1)
    packed, scales = orc.nf4_quantize(w, orc.F32, 64)
    assert np.array_equal(packed[:4096], z["codes_head"])
    assert hashlib.sha256(packed.tobytes()).hexdigest() == str(z["codes_sha256"])
    assert hashlib.sha256(scales.tobytes()).hexdigest() == str(z["scales_sha256"])
    wdeq = orc.nf4_dequantize(packed, scales, orc.F32).reshape(4096, 4096)
    y = orc.loralinear_forward(c1.X.numpy(), wdeq, None, c1.A.numpy(), c1.B.numpy(), c1.scaling, orc.F32)
    assert_matmul_close(y, z["y"], orc.F32)


def test_torch_port_matches_reference_layer():
    """oracle/torch_port.py (the timed CPU baseline) reproduces the
    reference's double-quant layer output on the golden case."""
    import torch
    from oracle import torch_port
    z = load("layers.npz")
    name = "nf4dq_bf16"
    c = _layer_case(z, name)
    N, K, M = c["N"], c["K"], c["M"]
    packed, scales = orc.nf4_quantize(z[f"{name}/w"], c["wdt"], 64)
    c2, c2s = orc.enable_double_quant(packed, scales, c["wdt"], N * K)
    x = torch.from_numpy(z[f"{name}/x"].astype(np.int16)).view(torch.bfloat16).reshape(M, K)
    A = torch.from_numpy(z[f"{name}/A"].reshape(c["r"], K))
    B = torch.from_numpy(z[f"{name}/B"].reshape(N, c["r"]))
    y = torch_port.loralinear_forward_dq(x, torch.from_numpy(packed), torch.from_numpy(c2), torch.from_numpy(c2s),
                                         N, K, A, B, c["alpha"] / c["r"])
    assert_matmul_close(y.float().numpy(), orc.to_f32(z[f"{name}/y"], 1).reshape(M, N), 1)
