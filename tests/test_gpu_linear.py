"""GPU parity of the fused QuantLinear + LoRA kernels (forward Y and dX).

Outputs are compared with the reference's own results (tests/golden/layers.npz,
config1.npz) and with the numpy oracle on seeded inputs, using the tolerance
of tests/tolerance.py: |y - y_ref| <= 1e-2 * RMS(y_ref) + 1 ulp (bf16 in,
fp32 accumulate).  Calls go through the package (which calls the C ABI) and,
for the raw-ABI cases, directly through ctypes.
"""
import ctypes
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import oracle as orc
from tests.gpu_util import from_bits, to_bits, to_f32
from tests.inputs import layer_inputs
from tests.tolerance import assert_matmul_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DTC = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")


def _golden_layers():
    z = np.load(os.path.join(GOLD, "layers.npz"))
    return z, sorted({k.rsplit("/", 1)[0] for k in z.files if k.endswith("/y")})


def build_layer(W, bits, dq, bias, r, alpha, A, B, block_size=64):
    """LoRALinear(QuantLinear.from_linear(...)) on the GPU, eval mode."""
    from rocm_qlora import LoRALinear, QuantLinear
    N, K = W.shape
    lin = nn.Linear(K, N, bias=bias is not None, device="cuda", dtype=W.dtype)
    with torch.no_grad():
        lin.weight.copy_(W.cuda())
        if bias is not None:
            lin.bias.copy_(bias.cuda())
    ql = QuantLinear.from_linear(lin, bits=bits, block_size=block_size)
    if dq:
        ql.enable_double_quant()
    lora = LoRALinear(ql, r=r, lora_alpha=alpha, lora_dropout=0.0).cuda().eval()
    with torch.no_grad():
        lora.lora_A.copy_(A.cuda())
        lora.lora_B.copy_(B.cuda())
    return lora


def oracle_wdeq(ql, N, K):
    """fp32 [N, K] dequantized weight recomputed by the oracle from the
    layer's own buffers."""
    q = to_bits(ql.weight_quant)
    if ql.bits == 4 and ql.use_double_quant:
        return orc.double_dequantize(q, to_bits(ql.c2).reshape(-1), to_bits(ql.c2_scales).reshape(-1),
                                     N * K).reshape(N, K)
    sdt = DTC[ql.weight_scales.dtype]
    if ql.bits == 4:
        return orc.nf4_dequantize(q, to_bits(ql.weight_scales).reshape(-1), sdt)[:N * K].reshape(N, K)
    return orc.int8_dequantize(q, to_bits(ql.weight_scales).reshape(-1), sdt)[:N * K].reshape(N, K)


@pytest.mark.parametrize("name", _golden_layers()[1])
def test_layer_golden(name):
    z, _ = _golden_layers()
    N, K, M, wdt, xdt, bits, has_bias, dq, r, alpha = (int(v) for v in z[f"{name}/meta"])
    W = from_bits(z[f"{name}/w"], wdt).reshape(N, K)
    bias = from_bits(z[f"{name}/bias"], wdt) if has_bias else None
    A = torch.from_numpy(z[f"{name}/A"]).reshape(r, K)
    B = torch.from_numpy(z[f"{name}/B"]).reshape(N, r)
    lora = build_layer(W, bits, dq, bias, r, alpha, A, B)
    assert np.array_equal(to_bits(lora.base_layer.weight_quant), z[f"{name}/qweight"])
    x = from_bits(z[f"{name}/x"], xdt).reshape(M, K).cuda().requires_grad_(True)
    dy = from_bits(z[f"{name}/dy"], xdt).reshape(M, N).cuda()
    y = lora(x)
    y.backward(dy)
    assert y.dtype == x.dtype
    assert_matmul_close(to_f32(y), orc.to_f32(z[f"{name}/y"], xdt).reshape(M, N), xdt)
    assert_matmul_close(to_f32(x.grad), orc.to_f32(z[f"{name}/dx"], xdt).reshape(M, K), xdt)


def _oracle_y_dx(lora, x, dy):
    ql = lora.base_layer
    N, K = ql.out_features, ql.in_features
    xdt = DTC[x.dtype]
    wdeq = oracle_wdeq(ql, N, K)
    A = lora.lora_A.detach().cpu().numpy()
    B = lora.lora_B.detach().cpu().numpy()
    bias = ql.bias.detach().float().cpu().numpy() if ql.bias is not None else None
    xf, dyf = to_f32(x), to_f32(dy)
    y = orc.loralinear_forward(xf, wdeq, bias, A, B, lora.scaling, xdt)
    dx = orc.loralinear_dx(dyf, wdeq, A, B, lora.scaling, xdt)
    return y, dx


@pytest.mark.parametrize("N,K", [(4096, 4096), (1000, 2048), (264, 11008), (600, 1088), (40, 320)])
@pytest.mark.parametrize("M", [1, 4, 5, 16])
def test_decode_gemv_nf4_dq_vs_oracle(N, K, M):
    """Decode shapes (GEMV path) with double-quantized NF4, r=16 alpha=32.
    K = 1088 and 320 are not multiples of 256 (the narrow code layout)."""
    inp = layer_inputs(N, K, M, sigma=0.02, r=16, alpha=32, seed=N + K + M, with_dy=True)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda().requires_grad_(True)
    y = lora(x)
    y.backward(inp.dY.cuda())
    y_ref, dx_ref = _oracle_y_dx(lora, inp.X, inp.dY)
    assert_matmul_close(to_f32(y), y_ref, 1)
    assert_matmul_close(to_f32(x.grad), dx_ref, 1)


@pytest.mark.parametrize("r", [8, 12, 3])
@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [1, 16])
def test_decode_gemv_lora_ranks(r, xdtype, M):
    """The decode GEMV's adapter epilogue for ranks that are a multiple of 8
    (16-byte loads of B and x.A^T) and ranks that are not (element loads)."""
    N, K = 600, 1024
    inp = layer_inputs(N, K, M, sigma=0.05, r=r, alpha=2 * r, w_dtype=xdtype, x_dtype=xdtype, seed=100 + r + M,
                       with_dy=True)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda().requires_grad_(True)
    y = lora(x)
    y.backward(inp.dY.cuda())
    y_ref, dx_ref = _oracle_y_dx(lora, inp.X, inp.dY)
    xdt = DTC[xdtype]
    assert_matmul_close(to_f32(y), y_ref, xdt)
    assert_matmul_close(to_f32(x.grad), dx_ref, xdt)


@pytest.mark.parametrize("fmt", ["nf4", "int8", "int8_row"])
@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [3, 16, 40])
def test_formats_dtypes_vs_oracle(fmt, xdtype, M):
    """NF4 / INT8 blockwise / INT8 per-row, bf16 and fp16 activations, with bias."""
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.quantization import quantize_int8
    N, K = 520, 1024
    inp = layer_inputs(N, K, M, sigma=0.05, r=8, alpha=16, w_dtype=xdtype, x_dtype=xdtype, seed=M, with_dy=True)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.1).to(xdtype)
    if fmt == "int8_row":
        ql = QuantLinear(K, N, bits=8, bias=True).cuda()
        q, s = quantize_int8(inp.W.cuda(), per_channel=True)
        ql.weight_quant, ql.weight_scales = q, s
        ql.bias = bias.cuda()
        lora = LoRALinear(ql, r=inp.r, lora_alpha=inp.alpha).cuda().eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A.cuda())
            lora.lora_B.copy_(inp.B.cuda())
        wdeq = orc.int8_dequantize(to_bits(q).reshape(-1), to_bits(s), DTC[xdtype], rows=N, cols=K).reshape(N, K)
    else:
        lora = build_layer(inp.W, 4 if fmt == "nf4" else 8, False, bias, inp.r, inp.alpha, inp.A, inp.B)
        wdeq = oracle_wdeq(lora.base_layer, N, K)
    x = inp.X.cuda().requires_grad_(True)
    y = lora(x)
    y.backward(inp.dY.cuda())
    xdt = DTC[xdtype]
    A, B = inp.A.numpy(), inp.B.numpy()
    y_ref = orc.loralinear_forward(to_f32(inp.X), wdeq, bias.float().numpy(), A, B, lora.scaling, xdt)
    dx_ref = orc.loralinear_dx(to_f32(inp.dY), wdeq, A, B, lora.scaling, xdt)
    assert_matmul_close(to_f32(y), y_ref, xdt)
    assert_matmul_close(to_f32(x.grad), dx_ref, xdt)


def test_config1_forward_golden():
    """Config 1: fp32 4096x4096 NF4, X 32x4096, r=16 alpha=32 -- Y against
    the reference's Y."""
    from tests.inputs import config1
    z = np.load(os.path.join(GOLD, "config1.npz"))
    c1 = config1()
    lora = build_layer(c1.W, 4, False, None, c1.r, c1.alpha, c1.A, c1.B)
    y = lora(c1.X.cuda())
    assert_matmul_close(to_f32(y), z["y"], 0)


def test_lora_grads_flow_and_match_torch():
    """dA and dB follow the reference autograd (bf16 matmuls of the same
    operands)."""
    inp = layer_inputs(256, 512, 8, sigma=0.05, r=8, alpha=16, seed=3, with_dy=True)
    lora = build_layer(inp.W, 4, False, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda()
    y = lora(x)
    y.backward(inp.dY.cuda())
    dy = inp.dY.cuda()
    A, B = lora.lora_A.detach().bfloat16(), lora.lora_B.detach().bfloat16()
    gu = dy * lora.scaling
    t = x @ A.t()
    gB = (gu.t() @ t).float()
    gA = ((gu @ B).t() @ x).float()
    torch.testing.assert_close(lora.lora_B.grad, gB, rtol=0, atol=0)
    torch.testing.assert_close(lora.lora_A.grad, gA, rtol=0, atol=0)


def test_zero_init_is_base_exactly():
    """B = 0 at init: LoRALinear output equals QuantLinear output bit for bit."""
    from rocm_qlora import LoRALinear, QuantLinear
    lin = nn.Linear(256, 128, device="cuda", dtype=torch.bfloat16)
    ql = QuantLinear.from_linear(lin, bits=4)
    lora = LoRALinear(ql, r=8).cuda()
    x = torch.randn(2, 256, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(lora(x), ql(x))


def test_dropout_training_path():
    """Train mode with LoRA dropout: forward/backward run, gradients reach
    x, A and B, and the base-only gradient matches eval mode when p -> the
    dropout mask is all ones (checked by comparing to a p=0 layer)."""
    from rocm_qlora import LoRALinear, QuantLinear
    torch.manual_seed(0)
    lin = nn.Linear(512, 256, device="cuda", dtype=torch.bfloat16)
    ql = QuantLinear.from_linear(lin, bits=4)
    lora = LoRALinear(ql, r=8, lora_dropout=0.1).cuda().train()
    with torch.no_grad():
        lora.lora_B.normal_()
    x = torch.randn(4, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = lora(x)
    y.float().sum().backward()
    assert x.grad is not None and lora.lora_A.grad.abs().sum() > 0 and lora.lora_B.grad.abs().sum() > 0


def test_merge_unmerge():
    from rocm_qlora import LoRALinear, QuantLinear
    torch.manual_seed(42)
    lin = nn.Linear(64, 128, device="cuda")
    ql = QuantLinear.from_linear(lin)
    lora = LoRALinear(ql, r=8).cuda()
    with torch.no_grad():
        lora.lora_A.normal_()
        lora.lora_B.normal_()
    x = torch.randn(2, 64, device="cuda")
    pre = lora(x)
    lora.merge_lora()
    post = lora(x)
    assert torch.allclose(post, pre, atol=2.0)
    assert lora.lora_A.abs().sum() == 0
    with pytest.raises(RuntimeError, match="LoRA already merged"):
        lora.merge_lora()
    lora.unmerge_lora()
    assert not ql.merged_mode


def test_fused_matmul_entry_points():
    """fused_dequant_nf4_matmul / fused_dequant_int8_matmul against dequantize + F.linear
    (reference tests/v2/test_kernels.py:51-68, block_size 32 and 64)."""
    from rocm_qlora.kernels import fused_dequant_int8_matmul, fused_dequant_nf4_matmul
    from rocm_qlora.quantization import quantize_int4, quantize_int8
    for bs in (32, 64):
        M, N, K = 4, 128, 256
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda")
        p, s = quantize_int4(w.flatten(), block_size=bs)
        y = fused_dequant_nf4_matmul(x, p.reshape(N, K // 2), s, block_size=bs)
        wdeq = orc.nf4_dequantize(p.cpu().numpy(), s.cpu().numpy(), 0, bs).reshape(N, K)
        assert_matmul_close(to_f32(y), orc.quantlinear_forward(to_f32(x), wdeq, None, 1), 1, roundings=1)
        q, s8 = quantize_int8(w.flatten(), block_size=bs)
        y8 = fused_dequant_int8_matmul(x, q.reshape(N, K), s8, block_size=bs)
        wdeq8 = orc.int8_dequantize(q.cpu().numpy(), s8.cpu().numpy(), 0, bs).reshape(N, K)
        assert_matmul_close(to_f32(y8), orc.quantlinear_forward(to_f32(x), wdeq8, None, 1), 1, roundings=1)
    x3 = torch.randn(2, 8, K, device="cuda", dtype=torch.bfloat16)
    assert fused_dequant_nf4_matmul(x3, p, s, block_size=64).shape == (2, 8, N)


def test_odd_shapes_exact_path():
    """37 x 73 (blocks straddle rows; reference tests/test_quant_linear.py:92-101)."""
    from rocm_qlora import QuantLinear
    for bits in (4, 8):
        lin = nn.Linear(37, 73, device="cuda")
        w = lin.weight.detach().clone()
        ql = QuantLinear.from_linear(lin, bits=bits, block_size=64)
        x = torch.randn(3, 37, device="cuda")
        y = ql(x)
        assert y.shape == (3, 73)
        wdeq = oracle_wdeq(ql, 73, 37)
        assert_matmul_close(to_f32(y), orc.quantlinear_forward(to_f32(x), wdeq, ql.bias.cpu().numpy(), 0), 0,
                            roundings=1)


def test_raw_abi_errors_and_drop_in_launcher():
    """Host-side validation through the raw C ABI, and the reference-named
    launcher launch_int4_dequant_matmul (fp16 x / scales / c)."""
    from rocm_qlora import _native as nat
    from rocm_qlora.quantization import quantize_int4
    L = nat.lib()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(4, 128, device="cuda", dtype=torch.bfloat16)
    q = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = torch.ones(2, device="cuda")
    y = torch.empty(4, 1, device="cuda", dtype=torch.bfloat16)
    # bad dtype code
    rc = L.rq_linear_forward(0, q.data_ptr(), s.data_ptr(), 0, None, None, 1, 128, 64, x.data_ptr(), 7, 4, None,
                             None, 0, None, None, 0, 1.0, y.data_ptr(), None, 0, st)
    assert rc == -3
    # misaligned activation pointer
    rc = L.rq_linear_forward(0, q.data_ptr(), s.data_ptr(), 0, None, None, 1, 128, 64, x.data_ptr() + 1, 1, 4, None,
                             None, 0, None, None, 0, 1.0, y.data_ptr(), None, 0, st)
    assert rc == -2
    # LoRA without workspace
    A = torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(1, 8, device="cuda", dtype=torch.bfloat16)
    rc = L.rq_linear_forward(0, q.data_ptr(), s.data_ptr(), 0, None, None, 1, 128, 64, x.data_ptr(), 1, 4, None,
                             None, 0, A.data_ptr(), B.data_ptr(), 8, 2.0, y.data_ptr(), None, 0, st)
    assert rc == -5
    # drop-in launcher with the reference's fp16 ABI
    M, N, K = 5, 256, 512
    xh = torch.randn(M, K, device="cuda", dtype=torch.float16)
    w = torch.randn(N, K, device="cuda", dtype=torch.float16) * 0.05
    p, sc = quantize_int4(w)
    c = torch.empty(M, N, device="cuda", dtype=torch.float16)
    L.launch_int4_dequant_matmul(st, xh.data_ptr(), p.data_ptr(), sc.data_ptr(), c.data_ptr(), M, N, K, 64)
    assert L.rq_last_status() == 0
    wdeq = orc.nf4_dequantize(p.cpu().numpy(), to_bits(sc), 2).reshape(N, K)
    assert_matmul_close(to_f32(c), orc.quantlinear_forward(to_f32(xh), wdeq, None, 2), 2, roundings=1)


def test_cuda_graph_capture_decode():
    """The decode path captures into a CUDA graph and replays correctly."""
    inp = layer_inputs(4096, 4096, 4, seed=9)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda()
    with torch.no_grad():
        y0 = lora(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lora(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yg = lora(x)
        g.replay()
        torch.cuda.synchronize()
    assert torch.equal(yg, y0)


@pytest.mark.parametrize("r,M", [(16, 1), (16, 16), (64, 5), (40, 16), (3, 2)])
def test_decode_fused_down_product(r, M):
    """The NF4 decode GEMV computes x.A^T in its own grid (down CTAs, a ready
    flag in the workspace counter area): parity with the oracle, identical
    results over back-to-back calls on one workspace (eager and replayed
    from a CUDA graph), and the counter area zero again afterwards."""
    from rocm_qlora import _native as nat
    N, K = 2304, 4096
    inp = layer_inputs(N, K, M, sigma=0.03, r=r, alpha=2 * r, seed=700 + r + M)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda()
    with torch.no_grad():
        y0 = lora(x)
        ys = [lora(x) for _ in range(8)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lora(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yg = lora(x)
        for _ in range(4):
            g.replay()
        torch.cuda.synchronize()
    y_ref, _ = _oracle_y_dx(lora, inp.X, torch.zeros(M, N, dtype=inp.X.dtype))
    assert_matmul_close(to_f32(y0), y_ref, 1, label=f"fused down product r{r} M{M}")
    assert all(torch.equal(y, y0) for y in ys) and torch.equal(yg, y0)
    ws = nat.workspace(torch.device("cuda", torch.cuda.current_device()), 0)
    assert int(ws[:256].count_nonzero()) == 0
    with torch.cuda.stream(s):
        ws_s = nat.workspace(torch.device("cuda", torch.cuda.current_device()), 0)
    assert int(ws_s[:256].count_nonzero()) == 0


@pytest.mark.parametrize("r,M", [(12, 64), (72, 300), (128, 40), (128, 256)])
def test_prefill_ranks_beside_the_gemm(r, M):
    """Ranks the tensor-core GEMM does not take (r > 64, r % 8 != 0) at
    prefill / training sizes: the kernel runs without the adapter and the
    adapter term is added with matmuls in the activation dtype; forward and
    dX keep the reference's roundings."""
    N, K = 512, 1024
    inp = layer_inputs(N, K, M, sigma=0.03, r=r, alpha=2 * r, seed=900 + r + M, with_dy=True)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    x = inp.X.cuda().requires_grad_(True)
    y = lora(x)
    y.backward(inp.dY.cuda())
    y_ref, dx_ref = _oracle_y_dx(lora, inp.X, inp.dY)
    assert_matmul_close(to_f32(y), y_ref, 1, label=f"rank {r} M{M} forward")
    assert_matmul_close(to_f32(x.grad), dx_ref, 1, label=f"rank {r} M{M} dx")


@pytest.mark.parametrize("M,r", [(4, 16), (300, 64), (96, 0)])
def test_torch_ops_equal_ctypes_calls(M, r):
    """torch.ops.rocm_qlora.* (the extension) and direct ctypes calls of the
    C ABI launch the same kernels: identical forward and dX bytes."""
    from rocm_qlora import _native as nat
    N, K = 640, 2048
    inp = layer_inputs(N, K, M, sigma=0.03, r=max(r, 1), alpha=32, seed=1200 + M + r, with_dy=True)
    lora = build_layer(inp.W, 4, True, None, inp.r, inp.alpha, inp.A, inp.B)
    assert nat.ops()

    def run():
        x = inp.X.cuda().requires_grad_(True)
        y = lora(x) if r else lora.base_layer(x)
        y.backward(inp.dY.cuda())
        torch.cuda.synchronize()
        return y.detach().clone(), x.grad.clone()

    y_ops, dx_ops = run()
    saved = nat._ops_state
    try:
        nat._ops_state = False
        y_ct, dx_ct = run()
    finally:
        nat._ops_state = saved
    assert torch.equal(y_ops, y_ct) and torch.equal(dx_ops, dx_ct)
