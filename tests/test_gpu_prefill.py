"""GPU parity of the tcgen05 prefill GEMM (M >= 64): forward Y of
QuantLinear / LoRALinear against the numpy oracle of the reference's eager
path, on seeded inputs, with the tolerance of tests/tolerance.py.  Each case
also checks that the tensor-core GEMM is the kernel that ran
(rq_last_path() == RQ_PATH_GEMM)."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.gpu_util import to_bits, to_f32
from tests.inputs import layer_inputs
from tests.test_gpu_linear import DTC, build_layer, oracle_wdeq
from tests.tolerance import assert_matmul_close

pytestmark = pytest.mark.gpu
RQ_PATH_GEMM = 2

CASES = [
    # N, K, M, r, double quant, dtype, bias
    (512, 1024, 64, 8, True, torch.bfloat16, False),
    (1000, 2048, 200, 16, True, torch.bfloat16, True),   # ragged N and M tiles
    (768, 512, 130, 0, False, torch.bfloat16, True),     # no adapter, plain bf16 scales
    (520, 1024, 256, 16, False, torch.float16, True),    # fp16 activations and scales
    (4096, 4096, 512, 64, True, torch.bfloat16, False),  # a configs[2] layer at M=512, r=64
    (4000, 512, 1200, 16, True, torch.bfloat16, True),   # 256-wide pair tiles (>= 148 CTAs), ragged N and M
]


@pytest.mark.parametrize("N,K,M,r,dq,dt,with_bias", CASES)
def test_prefill_gemm_vs_oracle(N, K, M, r, dq, dt, with_bias):
    from rocm_qlora import _native as nat
    inp = layer_inputs(N, K, M, sigma=0.02, r=max(r, 1), alpha=2 * max(r, 1), w_dtype=dt, x_dtype=dt,
                       seed=N + M + r)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(7)) * 0.1).to(dt) if with_bias else None
    lora = build_layer(inp.W, 4, dq, bias, max(r, 1), 2 * max(r, 1), inp.A, inp.B)
    layer = lora if r > 0 else lora.base_layer
    x = inp.X.cuda()
    with torch.no_grad():
        y = layer(x)
    torch.cuda.synchronize()
    assert nat.lib().rq_last_path() == RQ_PATH_GEMM
    c = ctypes_count(nat)
    assert c == 0, f"{c} bounded waits ran out"
    xdt = DTC[dt]
    wdeq = oracle_wdeq(lora.base_layer, N, K)
    bf = bias.float().numpy() if with_bias else None
    if r > 0:
        y_ref = orc.loralinear_forward(to_f32(inp.X), wdeq, bf, inp.A.numpy(), inp.B.numpy(), lora.scaling, xdt)
        assert_matmul_close(to_f32(y), y_ref, xdt, roundings=2)
    else:
        y_ref = orc.quantlinear_forward(to_f32(inp.X), wdeq, bf, xdt)
        assert_matmul_close(to_f32(y), y_ref, xdt, roundings=1)


DX_CASES = [
    # N, K, M, r, double quant, dtype
    (512, 1024, 64, 8, True, torch.bfloat16),
    (1024, 2048, 200, 16, True, torch.bfloat16),   # ragged M tile, K not a multiple of 256
    (640, 768, 130, 0, False, torch.float16),
    (4096, 4096, 512, 64, True, torch.bfloat16),
    (1024, 4032, 1200, 16, True, torch.bfloat16),  # 256-wide pair tiles, K tile past the last quant block
]


@pytest.mark.parametrize("N,K,M,r,dq,dt", DX_CASES)
def test_prefill_dx_gemm_vs_oracle(N, K, M, r, dq, dt):
    """Backward input gradient through the transposed tcgen05 GEMM."""
    from rocm_qlora import _native as nat
    inp = layer_inputs(N, K, M, sigma=0.02, r=max(r, 1), alpha=2 * max(r, 1), w_dtype=dt, x_dtype=dt,
                       seed=N + M + r + 1, with_dy=True)
    lora = build_layer(inp.W, 4, dq, None, max(r, 1), 2 * max(r, 1), inp.A, inp.B)
    layer = lora if r > 0 else lora.base_layer
    x = inp.X.cuda().requires_grad_(True)
    y = layer(x)
    y.backward(inp.dY.cuda())
    torch.cuda.synchronize()
    assert nat.lib().rq_last_path() == RQ_PATH_GEMM  # the dX call ran last
    assert ctypes_count(nat) == 0
    xdt = DTC[dt]
    wdeq = oracle_wdeq(lora.base_layer, N, K)
    if r > 0:
        dx_ref = orc.loralinear_dx(to_f32(inp.dY), wdeq, inp.A.numpy(), inp.B.numpy(), lora.scaling, xdt)
        assert_matmul_close(to_f32(x.grad), dx_ref, xdt, roundings=2)
    else:
        dx_ref = orc.loralinear_dx(to_f32(inp.dY), wdeq, None, None, 1.0, xdt)
        assert_matmul_close(to_f32(x.grad), dx_ref, xdt, roundings=1)


def ctypes_count(nat):
    import ctypes
    c = ctypes.c_uint(0)
    assert nat.lib().rq_take_kernel_timeouts(ctypes.byref(c)) == 0
    return c.value


def test_prefill_matches_decode_slabs_bitwise_free_of_state():
    """Two calls in a row give identical Y (no state carried between CTAs or
    calls)."""
    inp = layer_inputs(1024, 2048, 384, sigma=0.02, r=16, alpha=32, seed=3)
    lora = build_layer(inp.W, 4, True, None, 16, 32, inp.A, inp.B)
    x = inp.X.cuda()
    with torch.no_grad():
        y1 = lora(x).float().cpu().numpy()
        y2 = lora(x).float().cpu().numpy()
    assert np.array_equal(y1, y2)


@pytest.mark.parametrize("M", [300, 2048])
def test_prefill_dx_non_power_of_two_scaling(M):
    """dX with scaling 1.5: the tensor-core down product takes only power-of-
    two scales (exactness), so the other kernel computes gt = rnd(rnd(dY*s).B);
    the result stays within the tolerance of the reference."""
    from rocm_qlora import _native as nat
    N, K, r = 1024, 2048, 16
    inp = layer_inputs(N, K, M, sigma=0.02, r=r, alpha=24, w_dtype=torch.bfloat16, x_dtype=torch.bfloat16,
                       seed=M + 5, with_dy=True)
    lora = build_layer(inp.W, 4, True, None, r, 24, inp.A, inp.B)
    assert lora.scaling == 1.5
    x = inp.X.cuda().requires_grad_(True)
    lora(x).backward(inp.dY.cuda())
    torch.cuda.synchronize()
    assert nat.lib().rq_last_path() == RQ_PATH_GEMM
    assert ctypes_count(nat) == 0
    wdeq = oracle_wdeq(lora.base_layer, N, K)
    dx_ref = orc.loralinear_dx(to_f32(inp.dY), wdeq, inp.A.numpy(), inp.B.numpy(), lora.scaling, DTC[torch.bfloat16])
    assert_matmul_close(to_f32(x.grad), dx_ref, DTC[torch.bfloat16], roundings=2)


INT8_CASES = [
    # fmt, N, K, M, r, dtype
    ("int8", 520, 1024, 200, 16, torch.bfloat16),       # 128-wide pair tiles, ragged N and M
    ("int8_row", 1000, 2048, 130, 8, torch.float16),    # per-output-row scales
    ("int8", 4096, 1024, 1200, 16, torch.bfloat16),     # 256-wide pair tiles
]


@pytest.mark.parametrize("fmt,N,K,M,r,dt", INT8_CASES)
def test_prefill_int8_gemm_vs_oracle(fmt, N, K, M, r, dt):
    """INT8 weights (the reference's default bits=8, blockwise or per-row
    scales) through the tcgen05 GEMM: forward Y and dX against the oracle."""
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora import _native as nat
    from rocm_qlora.quantization import quantize_int8
    inp = layer_inputs(N, K, M, sigma=0.05, r=r, alpha=2 * r, w_dtype=dt, x_dtype=dt, seed=N + M, with_dy=True)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(9)) * 0.1).to(dt)
    if fmt == "int8_row":
        ql = QuantLinear(K, N, bits=8, bias=True).cuda()
        q, s = quantize_int8(inp.W.cuda(), per_channel=True)
        ql.weight_quant, ql.weight_scales = q, s
        ql.bias = bias.cuda()
        lora = LoRALinear(ql, r=r, lora_alpha=2 * r).cuda().eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A.cuda())
            lora.lora_B.copy_(inp.B.cuda())
        wdeq = orc.int8_dequantize(to_bits(q).reshape(-1), to_bits(s), DTC[dt], rows=N, cols=K).reshape(N, K)
    else:
        lora = build_layer(inp.W, 8, False, bias, r, 2 * r, inp.A, inp.B)
        wdeq = oracle_wdeq(lora.base_layer, N, K)
    x = inp.X.cuda().requires_grad_(True)
    y = lora(x)
    assert nat.lib().rq_last_path() == RQ_PATH_GEMM
    y.backward(inp.dY.cuda())
    torch.cuda.synchronize()
    assert nat.lib().rq_last_path() == RQ_PATH_GEMM
    assert ctypes_count(nat) == 0
    xdt = DTC[dt]
    A, B = inp.A.numpy(), inp.B.numpy()
    y_ref = orc.loralinear_forward(to_f32(inp.X), wdeq, bias.float().numpy(), A, B, lora.scaling, xdt)
    dx_ref = orc.loralinear_dx(to_f32(inp.dY), wdeq, A, B, lora.scaling, xdt)
    assert_matmul_close(to_f32(y), y_ref, xdt, roundings=2)
    assert_matmul_close(to_f32(x.grad), dx_ref, xdt, roundings=2)
