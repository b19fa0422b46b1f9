"""Generate the golden fixtures in tests/golden/ by running the REFERENCE.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_golden.py /path/to/ROCM-QLORA [state_dicts]

(the optional second argument writes only state_dicts.npz).

The reference package ``rocm_qlora`` is pure Python on torch.  Its ``.py``
sources are copied into a temporary directory (so no shipped bytecode is
loaded and nothing is written into the checkout), imported with
``ROCM_QLORA_QUIET=1``, and run on seeded CPU inputs.  Each fixture stores the
inputs and the reference's outputs as raw bit patterns (bf16/f16 as uint16,
fp8 as uint8) plus the torch version that produced them.

The fixtures pin both the C oracle (``-m "not gpu"`` tests) and the CUDA
kernels (``-m gpu`` tests) to the reference's own results.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import sys
import tempfile
import unittest.mock as mock

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.inputs import config1, layer_inputs  # noqa: E402


def _copy_reference(src: str, dst: str) -> None:
    for root, dirs, files in os.walk(src):
        dirs[:] = [d for d in dirs if d not in ("__pycache__", ".pytest_cache", ".git")]
        for f in files:
            if f.endswith(".py"):
                rel = os.path.relpath(root, src)
                os.makedirs(os.path.join(dst, rel), exist_ok=True)
                shutil.copy2(os.path.join(root, f), os.path.join(dst, rel, f))


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype in (torch.float8_e4m3fnuz, torch.float8_e4m3fn):
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_path: str, only: str = "") -> None:
    os.environ["ROCM_QLORA_QUIET"] = "1"
    sys.dont_write_bytecode = True
    tmp = tempfile.mkdtemp(prefix="rq_ref_")
    try:
        _copy_reference(ref_path, tmp)
        sys.path.insert(0, tmp)
        if only == "state_dicts":
            run_state_dicts()
        else:
            run(tmp)
            run_state_dicts()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def run_state_dicts() -> None:
    """state_dicts.npz: LoRALinear(QuantLinear) state dicts written by the
    reference (every tensor's bits and dtype under its state_dict key) with
    an input and the reference's eval-mode output, so that loading a
    reference checkpoint into this package can be checked."""
    import torch.nn as nn
    from rocm_qlora.quantization.quant_linear import QuantLinear
    from rocm_qlora.lora.lora_layer import LoRALinear
    out = {}
    for name, N, K, M, bits_, bias, dq_ in (("nf4_bias", 192, 512, 4, 4, True, False),
                                           ("nf4dq", 256, 1024, 8, 4, False, True),
                                           ("int8", 160, 512, 3, 8, True, False)):
        inp = layer_inputs(N, K, M, sigma=0.05, r=8, alpha=16, seed=N + K)
        lin = nn.Linear(K, N, bias=bias).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(inp.W)
            if bias:
                lin.bias.copy_((torch.randn(N, generator=torch.Generator().manual_seed(N)) * 0.1).to(torch.bfloat16))
        ql = QuantLinear.from_linear(lin, bits=bits_, block_size=64)
        if dq_:
            ql.enable_double_quant()
        lora = LoRALinear(ql, r=8, lora_alpha=16, lora_dropout=0.0).eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A)
            lora.lora_B.copy_(inp.B)
            y = lora(inp.X)
        for k, t in lora.state_dict().items():
            out[f"{name}/sd/{k}"] = bits(t)
            out[f"{name}/dtype/{k}"] = np.array(str(t.dtype).replace("torch.", ""))
        out[f"{name}/meta"] = np.array([N, K, M, bits_, int(bias), int(dq_)])
        out[f"{name}/x"], out[f"{name}/y"] = bits(inp.X), bits(y)
    out["torch"] = np.array(torch.__version__)
    np.savez_compressed(os.path.join(HERE, "state_dicts.npz"), **out)
    print("wrote state_dicts.npz with torch", torch.__version__)


def run(tmp: str) -> None:
    import torch.nn as nn
    from rocm_qlora.quantization import quant_ops as qo
    from rocm_qlora.quantization import double_quant as dq
    from rocm_qlora.quantization.quant_linear import QuantLinear
    from rocm_qlora.lora.lora_layer import LoRALinear

    meta = {"torch": torch.__version__}
    g = torch.Generator().manual_seed(1234)

    # ---------------------------------------------------------------- NF4
    nf4 = {}
    cases = []
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        for bs in (32, 64, 128):
            for n in (1000, 4096):
                x = (torch.randn(n, generator=g) * 0.05).to(dtype)
                cases.append((f"rand_{DT[dtype]}_{bs}_{n}", x, bs))
        # edge values: an all-zero block, exact table points, midpoints
        # between neighbouring levels (ties go to the lower index), tiny and
        # huge magnitudes, and a NaN / inf block.
        T = torch.tensor(qo.NF4_VALUES, dtype=torch.float32)
        mids = ((T[1:] + T[:-1]) / 2)
        edge = torch.cat([
            torch.zeros(64),
            T.repeat(4),
            torch.cat([mids, torch.tensor([1.0])]).repeat(4),
            torch.cat([mids * 3.0, torch.tensor([3.0])]).repeat(4),
            torch.randn(64, generator=g) * 1e-30,
            torch.randn(64, generator=g) * 1e30 if dtype != torch.float16 else torch.randn(64, generator=g) * 1e4,
            torch.randn(64, generator=g),
        ])
        cases.append((f"edge_{DT[dtype]}", edge.to(dtype), 64))
        special = torch.randn(128, generator=g)
        special[3] = float("nan")
        special[64 + 5] = float("inf")
        cases.append((f"special_{DT[dtype]}", special.to(dtype), 64))
    for name, x, bs in cases:
        p, s = qo.quantize_int4(x, block_size=bs)
        d = qo.dequantize_int4(p, s, block_size=bs)
        nf4[f"{name}/x"] = bits(x)
        nf4[f"{name}/dtype"] = np.int32(DT[x.dtype])
        nf4[f"{name}/bs"] = np.int32(bs)
        nf4[f"{name}/packed"] = bits(p)
        nf4[f"{name}/scales"] = bits(s.reshape(-1))
        nf4[f"{name}/deq"] = bits(d)
    nf4["table"] = np.array(qo.NF4_VALUES, dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "nf4.npz"), **nf4, **{"meta/torch": meta["torch"]})

    # --------------------------------------------------------------- INT8
    i8 = {}
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        for bs in (32, 64):
            x = (torch.randn(1000, generator=g) * 0.05).to(dtype)
            x[0] = 3.0
            q, s = qo.quantize_int8(x, block_size=bs)
            d = qo.dequantize_int8(q, s, block_size=bs)
            k = f"block_{DT[dtype]}_{bs}"
            i8[f"{k}/x"], i8[f"{k}/dtype"], i8[f"{k}/bs"] = bits(x), np.int32(DT[dtype]), np.int32(bs)
            i8[f"{k}/q"], i8[f"{k}/scales"], i8[f"{k}/deq"] = bits(q), bits(s.reshape(-1)), bits(d)
        w = (torch.randn(48, 200, generator=g) * 0.02).to(dtype)
        w[3] = 0.0
        q, s = qo.quantize_int8(w, per_channel=True)
        d = qo.dequantize_int8(q, s)
        k = f"rows_{DT[dtype]}"
        i8[f"{k}/x"], i8[f"{k}/dtype"] = bits(w), np.int32(DT[dtype])
        i8[f"{k}/q"], i8[f"{k}/scales"], i8[f"{k}/deq"] = bits(q), bits(s), bits(d)
    # bf16 blocks where round(x/scale) reaches 128 and wraps to -128 in the
    # reference's float->int8 cast: search a seeded stream for such blocks.
    gw = torch.Generator().manual_seed(7)
    found = []
    while len(found) < 4:
        a = (torch.randn(64, generator=gw) * float(torch.rand(1, generator=gw) * 100)).to(torch.bfloat16)
        s = a.abs().max() / 127.0
        if torch.round(a / s).abs().max() > 127:
            found.append(a)
    x = torch.cat(found)
    q, s = qo.quantize_int8(x, block_size=64)
    i8["wrap/x"], i8["wrap/dtype"], i8["wrap/bs"] = bits(x), np.int32(1), np.int32(64)
    i8["wrap/q"], i8["wrap/scales"] = bits(q), bits(s.reshape(-1))
    np.savez_compressed(os.path.join(HERE, "int8.npz"), **i8)

    # ------------------------------------------------------ double quant
    dqf = {}
    # the API path: QuantLinear.from_linear(bits=4) + enable_double_quant()
    for dtype, (N, K) in ((torch.bfloat16, (96, 320)), (torch.float32, (16, 4096)),
                          (torch.bfloat16, (8, 64 * 300))):
        lin = nn.Linear(K, N, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        lin = lin.to(dtype)
        w = lin.weight.detach().clone()
        ql = QuantLinear.from_linear(lin, bits=4, block_size=64)
        packed0, scales0 = ql.weight_quant.clone(), ql.weight_scales.clone()
        ok = ql.enable_double_quant()
        assert ok
        W_dd = dq.double_dequantize(dq.DoubleQuantState(
            W_quant=ql.weight_quant, c2=ql.c2, c2_scales=ql.c2_scales, blocksize_1=64,
            blocksize_2=256, original_shape=ql.original_shape, use_fp8_c2=ql.use_fp8_c2))
        k = f"api_{DT[dtype]}_{N}x{K}"
        dqf[f"{k}/w"], dqf[f"{k}/dtype"], dqf[f"{k}/shape"] = bits(w), np.int32(DT[dtype]), np.array([N, K])
        dqf[f"{k}/packed"], dqf[f"{k}/scales"] = bits(packed0), bits(scales0)
        dqf[f"{k}/c2"], dqf[f"{k}/c2_scales"] = bits(ql.c2), bits(ql.c2_scales.reshape(-1))
        dqf[f"{k}/deq"] = bits(W_dd)
    # double_quantize called directly, fp8 and the INT8 fallback
    for fp8 in (True, False):
        W = torch.randn(100, 200, generator=g) * 0.02
        W[0, :64] = 0.0
        if fp8:
            st = dq.double_quantize(W)
        else:
            with mock.patch("rocm_qlora.quantization.double_quant._has_fp8", return_value=False):
                st = dq.double_quantize(W)
        k = f"direct_{int(fp8)}"
        dqf[f"{k}/w"], dqf[f"{k}/packed"] = bits(W), bits(st.W_quant)
        dqf[f"{k}/c2"], dqf[f"{k}/c2_scales"] = bits(st.c2), bits(st.c2_scales.reshape(-1))
        dqf[f"{k}/deq"] = bits(dq.double_dequantize(st))
    # e4m3fnuz: every code decoded, and a sweep of fp32 values encoded
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fnuz)
    dqf["fp8/decode"] = bits(codes.to(torch.float32))
    sweep = torch.cat([torch.linspace(0, 1, 4097), torch.logspace(-14, 0, 2049, base=2.0),
                       -torch.linspace(0, 1, 257), torch.tensor([240.0, 244.0, 247.9, 248.0, 300.0])])
    dqf["fp8/sweep"] = bits(sweep)
    dqf["fp8/encode"] = bits(sweep.to(torch.float8_e4m3fnuz))
    np.savez_compressed(os.path.join(HERE, "double_quant.npz"), **dqf)

    # -------------------------------------------------- layer outputs
    lay = {}

    def layer_case(name, N, K, M, w_dtype, x_dtype, bits_, bias, dq_, r=8, alpha=16, seed=0):
        inp = layer_inputs(N, K, M, sigma=0.05, r=r, alpha=alpha, w_dtype=w_dtype,
                           x_dtype=x_dtype, seed=seed, with_dy=True)
        lin = nn.Linear(K, N, bias=bias).to(w_dtype)
        with torch.no_grad():
            lin.weight.copy_(inp.W)
            if bias:
                lin.bias.copy_((torch.randn(N, generator=g) * 0.1).to(w_dtype))
        b = lin.bias.detach().clone() if bias else None
        ql = QuantLinear.from_linear(lin, bits=bits_, block_size=64)
        if dq_:
            ql.enable_double_quant()
        lora = LoRALinear(ql, r=r, lora_alpha=alpha, lora_dropout=0.0).eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A)
            lora.lora_B.copy_(inp.B)
        x = inp.X.clone().requires_grad_(True)
        y = lora(x)
        y.backward(inp.dY)
        lay[f"{name}/w"], lay[f"{name}/x"], lay[f"{name}/dy"] = bits(inp.W), bits(inp.X), bits(inp.dY)
        lay[f"{name}/A"], lay[f"{name}/B"] = bits(inp.A), bits(inp.B)
        lay[f"{name}/meta"] = np.array([N, K, M, DT[w_dtype], DT[x_dtype], bits_, int(bias), int(dq_), r, alpha])
        if bias:
            lay[f"{name}/bias"] = bits(b)
        lay[f"{name}/qweight"] = bits(ql.weight_quant)
        lay[f"{name}/scales"] = bits(ql.weight_scales)
        if dq_:
            lay[f"{name}/c2"], lay[f"{name}/c2_scales"] = bits(ql.c2), bits(ql.c2_scales.reshape(-1))
        lay[f"{name}/y"] = bits(y)
        lay[f"{name}/dx"] = bits(x.grad)

    layer_case("nf4_f32", 128, 256, 4, torch.float32, torch.float32, 4, True, False)
    layer_case("nf4_bf16", 192, 320, 5, torch.bfloat16, torch.bfloat16, 4, False, False)
    layer_case("nf4dq_bf16", 256, 512, 16, torch.bfloat16, torch.bfloat16, 4, False, True, r=16, alpha=32)
    layer_case("nf4dq_bf16_bias", 128, 1024, 3, torch.bfloat16, torch.bfloat16, 4, True, True)
    layer_case("int8_bf16", 160, 256, 7, torch.bfloat16, torch.bfloat16, 8, True, False)
    layer_case("nf4_f16", 128, 256, 4, torch.float16, torch.float16, 4, False, False)
    layer_case("nf4dq_bf16_m130", 128, 256, 130, torch.bfloat16, torch.bfloat16, 4, False, True, r=64, alpha=128)
    np.savez_compressed(os.path.join(HERE, "layers.npz"), **lay)

    # ---------------------------------------------------- config 1 pins
    c1 = config1()
    p, s = qo.quantize_int4(c1.W.flatten(), block_size=64)
    lin = nn.Linear(4096, 4096, bias=False)
    with torch.no_grad():
        lin.weight.copy_(c1.W)
    ql = QuantLinear.from_linear(lin, bits=4, block_size=64)
    assert torch.equal(ql.weight_quant, p)
    lora = LoRALinear(ql, r=c1.r, lora_alpha=c1.alpha, lora_dropout=0.0).eval()
    with torch.no_grad():
        lora.lora_A.copy_(c1.A)
        lora.lora_B.copy_(c1.B)
        y = lora(c1.X)
    cfg = {
        "codes_sha256": sha(bits(p)),
        "scales_sha256": sha(bits(s)),
        "y": bits(y),
        "codes_head": bits(p)[:4096],
        "scales_head": bits(s)[:1024],
        "torch": meta["torch"],
    }
    np.savez_compressed(os.path.join(HERE, "config1.npz"), **cfg)
    print("wrote fixtures with torch", meta["torch"])


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: make_golden.py <path to the ROCM-QLORA checkout> [state_dicts]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) == 3 else "")
