"""GPU parity on the exact configurations bench.py reports.

* Decode: the three Llama-2-7B projections at M in {1, 4, 16},
  NF4 with double-quantized scales, LoRA r16 alpha 32, built as the bench
  builds them.
* 70B-shaped decode (configs[4] on one GPU): W 8192x28672 and 28672x8192 at
  M in {1, 16}, NF4 + double quant with and without the adapter, and INT8
  with per-row scales.  These layers give each CTA of the decode GEMV more
  rows than one pass holds, so the multi-pass form (per-pass scale staging,
  separate partial-sum region) is what runs.  The oracle works on row
  slices of the weight so that the reference result fits in host memory.
* Prefill / training: forward Y and backward dX of the three 7B
  projections at M in {512, 2048, 8192}, r64 alpha 128.  Output rows depend
  only on their own input rows, so the oracle checks a fixed sample of rows
  spread over every token tile (first, last, tile edges, random).

Every check records its plain max-abs / RMS figure and how many outputs
needed the ulp allowance of tests/tolerance.py; the session prints them.
References: quant_linear.py:159-197 (dequantize + F.linear),
lora_layer.py:51-70 (the adapter), double_quant.py:99-122 (double
dequantization), kernels/dequant_matmul.py:337-351 (dX).
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import oracle as orc
from tests.gpu_util import to_bits, to_f32
from tests.inputs import DECODE_M, DECODE_SHAPES, PREFILL_M, layer_inputs
from tests.tolerance import assert_matmul_close

pytestmark = pytest.mark.gpu
BF16 = 1
RQ_PATH_GEMV, RQ_PATH_GEMM = 1, 2


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")


def _lib():
    from rocm_qlora import _native as nat
    return nat.lib()


def _no_timeouts():
    import ctypes
    c = ctypes.c_uint(0)
    assert _lib().rq_take_kernel_timeouts(ctypes.byref(c)) == 0
    assert c.value == 0, f"{c.value} bounded in-kernel waits ran out"


def _nf4_dq_layer(W, r, alpha, A, B):
    from rocm_qlora import LoRALinear, QuantLinear
    N, K = W.shape
    lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        lin.weight.copy_(W.cuda())
    ql = QuantLinear.from_linear(lin, bits=4)
    ql.enable_double_quant()
    del lin
    lora = LoRALinear(ql, r=r, lora_alpha=alpha).cuda().eval()
    with torch.no_grad():
        lora.lora_A.copy_(A.cuda())
        lora.lora_B.copy_(B.cuda())
    return lora


class RowOracle:
    """Dequantized rows [r0, r1) of a QuantLinear's weight (fp32), computed by
    the oracle from the layer's own buffers without materialising the whole
    weight."""

    def __init__(self, ql):
        self.N, self.K = ql.out_features, ql.in_features
        self.q = to_bits(ql.weight_quant).reshape(-1)
        self.dq = ql.bits == 4 and getattr(ql, "use_double_quant", False)
        if self.dq:
            nb = self.N * self.K // 64
            self.c1 = orc.dq_first_level(to_bits(ql.c2).reshape(-1), to_bits(ql.c2_scales).reshape(-1), nb)
        else:
            self.s = to_bits(ql.weight_scales).reshape(-1)
            self.sdt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[ql.weight_scales.dtype]
        self.bits = ql.bits

    def rows(self, r0, r1):
        K = self.K
        if self.bits == 4 and self.dq:
            p = self.q[r0 * K // 2:r1 * K // 2]
            return orc.nf4_dequantize(p, self.c1[r0 * K // 64:r1 * K // 64], 0, 64).reshape(r1 - r0, K)
        if self.bits == 4:
            p = self.q[r0 * K // 2:r1 * K // 2]
            return orc.nf4_dequantize(p, self.s[r0 * K // 64:r1 * K // 64], self.sdt, 64).reshape(r1 - r0, K)
        q = self.q[r0 * K:r1 * K]
        return orc.int8_dequantize(q, self.s[r0:r1], self.sdt, rows=r1 - r0, cols=K).reshape(r1 - r0, K)


def _oracle_forward(ql, x_f32, A, B, scaling, chunk=2048):
    """y[M, N] of LoRALinear.forward (eval) over the layer's buffers, over
    row chunks of W (columns of y)."""
    ro = RowOracle(ql)
    N = ro.N
    out = np.empty((x_f32.shape[0], N), np.float32)
    for r0 in range(0, N, chunk):
        r1 = min(N, r0 + chunk)
        w = ro.rows(r0, r1)
        if A is None:
            out[:, r0:r1] = orc.quantlinear_forward(x_f32, w, None, BF16)
        else:
            out[:, r0:r1] = orc.loralinear_forward(x_f32, w, None, A, B[r0:r1], scaling, BF16)
    return out


# ------------------------------------------------------------ 7B decode

@pytest.mark.parametrize("si", range(len(DECODE_SHAPES)))
def test_bench_decode_7b(si):
    """configs[1] exactly as bench.py builds it (seed 100 + shape index):
    the three layers at M = 1, 4, 16 with the adapter."""
    N, K = DECODE_SHAPES[si]
    inp = layer_inputs(N, K, 1, sigma=0.02, r=16, alpha=32, seed=100 + si)
    lora = _nf4_dq_layer(inp.W, 16, 32, inp.A, inp.B)
    A, B = inp.A.numpy(), inp.B.numpy()
    g = torch.Generator().manual_seed(7)
    for M in DECODE_M:
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            y = lora(x.cuda())
        torch.cuda.synchronize()
        assert _lib().rq_last_path() == RQ_PATH_GEMV
        _no_timeouts()
        y_ref = _oracle_forward(lora.base_layer, to_f32(x), A, B, lora.scaling)
        assert_matmul_close(to_f32(y), y_ref, BF16, roundings=2, label=f"decode {N}x{K} M{M} r16")


# ---------------------------------------------------- 70B decode (multi-pass)

SHAPES_70B = [(8192, 28672), (28672, 8192)]


def _w70(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.015).to(torch.bfloat16)
    A = (torch.rand(16, K, generator=g) * 2 - 1) / K ** 0.5
    B = torch.randn(N, 16, generator=g) * 0.01
    return W, A, B


@pytest.mark.parametrize("N,K", SHAPES_70B)
def test_bench_decode_70b_nf4_dq(N, K):
    """NF4 + double quant at the 70B shapes, M in {1, 16}, with and without
    the adapter (the multi-pass decode GEMV); plus the quantization itself on
    a row slice whose double-quant groups straddle rows when K = 28672."""
    W, A, B = _w70(N, K, seed=N + 3)
    lora = _nf4_dq_layer(W, 16, 32, A, B)
    ql = lora.base_layer

    # codes and second level of rows [4096, 4160) against the oracle
    r0, r1 = 4096, 4160
    wsl = W[r0:r1].contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    packed, scales = orc.nf4_quantize(wsl, BF16, 64)
    assert np.array_equal(to_bits(ql.weight_quant).reshape(-1)[r0 * K // 2:r1 * K // 2], packed)
    c2, c2s = orc.enable_double_quant(packed, scales, BF16, (r1 - r0) * K)
    g0, g1 = r0 * K // 64 // 256, r1 * K // 64 // 256
    assert (r0 * K // 64) % 256 == 0 and (r1 * K // 64) % 256 == 0
    assert np.array_equal(to_bits(ql.c2).reshape(-1)[g0 * 256:g1 * 256], c2[:(g1 - g0) * 256])
    assert np.array_equal(to_bits(ql.c2_scales).reshape(-1)[g0:g1].view(np.uint32), c2s[:g1 - g0].view(np.uint32))

    An, Bn = A.numpy(), B.numpy()
    g = torch.Generator().manual_seed(N)
    for M in (1, 16):
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            y = lora(x.cuda())
            y0 = ql(x.cuda())
        torch.cuda.synchronize()
        assert _lib().rq_last_path() == RQ_PATH_GEMV
        _no_timeouts()
        xf = to_f32(x)
        y_ref = _oracle_forward(ql, xf, An, Bn, lora.scaling)
        assert_matmul_close(to_f32(y), y_ref, BF16, roundings=2, label=f"decode 70B {N}x{K} M{M} nf4-dq r16")
        y0_ref = _oracle_forward(ql, xf, None, None, 1.0)
        assert_matmul_close(to_f32(y0), y0_ref, BF16, roundings=1, label=f"decode 70B {N}x{K} M{M} nf4-dq base")


@pytest.mark.parametrize("N,K", SHAPES_70B)
def test_bench_decode_70b_int8_row(N, K):
    """INT8 with per-row scales (quantize_int8(per_channel=True)) at the 70B
    shapes, M in {1, 16}, with the adapter."""
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.quantization import quantize_int8
    W, A, B = _w70(N, K, seed=N + 5)
    ql = QuantLinear(K, N, bits=8, bias=False).cuda()
    q, s = quantize_int8(W.cuda(), per_channel=True)
    ql.weight_quant, ql.weight_scales = q, s
    # quantization bits of a row slice against the oracle
    r0, r1 = 1000, 1040
    wsl = W[r0:r1].contiguous().view(torch.int16).numpy().view(np.uint16)
    oq, os_ = orc.int8_quantize_rows(wsl, BF16)
    assert np.array_equal(to_bits(q)[r0:r1].reshape(-1), oq.reshape(-1))
    assert np.array_equal(to_bits(s).reshape(-1)[r0:r1], os_.reshape(-1))
    lora = LoRALinear(ql, r=16, lora_alpha=32).cuda().eval()
    with torch.no_grad():
        lora.lora_A.copy_(A.cuda())
        lora.lora_B.copy_(B.cuda())
    g = torch.Generator().manual_seed(N + 1)
    for M in (1, 16):
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            y = lora(x.cuda())
        torch.cuda.synchronize()
        assert _lib().rq_last_path() == RQ_PATH_GEMV
        _no_timeouts()
        y_ref = _oracle_forward(ql, to_f32(x), A.numpy(), B.numpy(), lora.scaling)
        assert_matmul_close(to_f32(y), y_ref, BF16, roundings=2, label=f"decode 70B {N}x{K} M{M} int8-row r16")


# ---------------------------------------------------------- 7B prefill / dX

def _sample_rows(M, seed):
    rng = np.random.default_rng(seed)
    fixed = [0, 1, 127, 128, 255, 256, M // 2, M - 257, M - 256, M - 129, M - 128, M - 1]
    rest = rng.choice(M, size=52, replace=False)
    return np.array(sorted({int(v) for v in fixed + list(rest) if 0 <= v < M}))


@pytest.mark.parametrize("si", range(len(DECODE_SHAPES)))
def test_bench_prefill_7b(si):
    """configs[2] as bench.py builds it (seed 200 + shape index, r64
    alpha 128): forward and dX at M = 512, 2048, 8192 on the tcgen05 GEMM."""
    N, K = DECODE_SHAPES[si]
    inp = layer_inputs(N, K, 1, sigma=0.02, r=64, alpha=128, seed=200 + si)
    lora = _nf4_dq_layer(inp.W, 64, 128, inp.A, inp.B)
    ql = lora.base_layer
    ro = RowOracle(ql)
    wdeq = ro.rows(0, N)
    A, B = inp.A.numpy(), inp.B.numpy()
    g = torch.Generator().manual_seed(si)
    for M in PREFILL_M:
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
        xc = x.cuda().requires_grad_(True)
        y = lora(xc)
        torch.cuda.synchronize()
        y_rows = to_f32(y)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        assert _lib().rq_last_path() == RQ_PATH_GEMM  # dX ran on the tensor-core GEMM
        _no_timeouts()
        rows = _sample_rows(M, seed=M + si)
        xs, dys = to_f32(x)[rows], to_f32(dy)[rows]
        y_ref = orc.loralinear_forward(xs, wdeq, None, A, B, lora.scaling, BF16)
        assert_matmul_close(y_rows[rows], y_ref, BF16, roundings=2, label=f"prefill fwd {N}x{K} M{M} r64")
        dx_ref = orc.loralinear_dx(dys, wdeq, A, B, lora.scaling, BF16)
        assert_matmul_close(to_f32(xc.grad)[rows], dx_ref, BF16, roundings=2, label=f"prefill dX {N}x{K} M{M} r64")
        del x, dy, xc, y


# ------------------------------------------ activations that share a sign

@pytest.fixture
def decode_mode():
    from rocm_qlora import _native as nat
    yield nat.set_decode_exact
    nat.set_decode_exact(False)


@pytest.mark.parametrize("exact", [True, False])
def test_decode_relu_inputs(exact, decode_mode):
    """Non-negative activations (as after a ReLU) on a 7B-shaped layer
    (4096 x 11008, M = 16, NF4 + double quant).  The exact decode numerics
    form the reference's own weights and meet the bar.  The default numerics
    round each level once, a fixed error per code that adds up over K when
    the activations share a sign: that figure (6.3e-2 x RMS on B200) is
    recorded and held to 8e-2 x RMS so that a regression shows.  (For scale: the reference's own
    rounding of level x scale moves these outputs by up to ~2.4e-2 x RMS
    from the unrounded product.)"""
    decode_mode(exact)
    N, K, M = 4096, 11008, 16
    inp = layer_inputs(N, K, 1, sigma=0.02, r=16, alpha=32, seed=300)
    lora = _nf4_dq_layer(inp.W, 16, 32, inp.A, inp.B)
    ql = lora.base_layer
    x = torch.relu(torch.randn(M, K, generator=torch.Generator().manual_seed(301))).to(torch.bfloat16)
    with torch.no_grad():
        y = ql(x.cuda())
    torch.cuda.synchronize()
    assert _lib().rq_last_path() == RQ_PATH_GEMV
    _no_timeouts()
    y_ref = _oracle_forward(ql, to_f32(x), None, None, 1.0)
    label = f"decode {N}x{K} M{M} relu inputs, {'exact' if exact else 'default'} numerics"
    if exact:
        assert_matmul_close(to_f32(y), y_ref, BF16, roundings=1, label=label)
    else:
        err = np.abs(to_f32(y).astype(np.float64) - y_ref).max() / np.sqrt(np.mean(y_ref.astype(np.float64) ** 2))
        from tests.tolerance import RECORDED
        RECORDED.append((label, float(err), -1, y_ref.size))
        assert err <= 8e-2, f"max-abs / RMS {err:.4f}"


@pytest.mark.parametrize("si", range(len(DECODE_SHAPES)))
def test_bench_decode_7b_exact(si, decode_mode):
    """configs[1] with the exact decode numerics."""
    decode_mode(True)
    N, K = DECODE_SHAPES[si]
    inp = layer_inputs(N, K, 1, sigma=0.02, r=16, alpha=32, seed=100 + si)
    lora = _nf4_dq_layer(inp.W, 16, 32, inp.A, inp.B)
    g = torch.Generator().manual_seed(7)
    for M in DECODE_M:
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            y = lora(x.cuda())
        torch.cuda.synchronize()
        assert _lib().rq_last_path() == RQ_PATH_GEMV
        _no_timeouts()
        y_ref = _oracle_forward(lora.base_layer, to_f32(x), inp.A.numpy(), inp.B.numpy(), lora.scaling)
        assert_matmul_close(to_f32(y), y_ref, BF16, roundings=2, label=f"decode {N}x{K} M{M} r16 exact")
