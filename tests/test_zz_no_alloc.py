"""rq_linear_forward_noalloc: the layer forward for callers that cannot
allocate device memory (plugin hosts that own all device memory, cgo / JNI /
FFI bindings without a CUDA allocator, loops where cudaMalloc would
synchronize the device).

The entry point takes its scratch from a fixed array inside the library.
These tests call it through the C ABI and compare it with rq_linear_forward
(given an ordinary workspace) on two calls in a row, so that leftovers of
the first call in the shared array would show up in the second.  The file
is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

from tests.inputs import layer_inputs
from tests.tolerance import assert_matmul_close

pytestmark = pytest.mark.gpu

RQ_ERR_SCRATCH = -7
SCRATCH_BYTES = 2 << 20


@pytest.fixture(scope="module")
def lib():
    from rocm_qlora import _native as nat
    if not nat.is_available():
        pytest.fail("B200 kernels unavailable on this machine")
    return nat.lib()


def _layer(N, K, r, seed):
    from rocm_qlora import LoRALinear, QuantLinear
    inp = layer_inputs(N, K, 1, sigma=0.02, r=r, alpha=2 * r, seed=seed)
    lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        lin.weight.copy_(inp.W.cuda())
    ql = QuantLinear.from_linear(lin, bits=4)
    ql.enable_double_quant()
    lora = LoRALinear(ql, r=r, lora_alpha=2 * r).cuda().eval()
    with torch.no_grad():
        lora.lora_A.copy_(inp.A.cuda())
        lora.lora_B.copy_(inp.B.cuda())
    return lora


def _forward(lib, lora, x, noalloc):
    from rocm_qlora import _native as nat
    w = lora.base_layer.weight_view()
    A = lora.lora_A.detach().bfloat16().contiguous()
    B = lora.lora_B.detach().bfloat16().contiguous()
    M = x.shape[0]
    y = torch.empty(M, w.N, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    if noalloc:
        rc = lib.rq_linear_forward_noalloc(*w.args(), x.data_ptr(), nat.BF16, M, None, None, 0, A.data_ptr(),
                                           B.data_ptr(), A.shape[0], float(lora.scaling), y.data_ptr(), st)
    else:
        nbytes = lib.rq_linear_workspace_bytes(M, w.N, w.K, A.shape[0])
        ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.rq_linear_forward(*w.args(), x.data_ptr(), nat.BF16, M, None, None, 0, A.data_ptr(), B.data_ptr(),
                                   A.shape[0], float(lora.scaling), y.data_ptr(), ws.data_ptr(), ws.numel(), st)
    assert rc == 0, lib.rq_status_string(rc)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


# r = 96 with M <= 16 takes the split-K down product whose arrival counters
# live in the scratch's first 256 bytes: the second call shows whether the
# per-call clearing and the kernels' reset of the counters hold.
@pytest.mark.parametrize("N,K,M,r", [(1024, 2048, 4, 16), (4096, 4096, 16, 16), (520, 1024, 40, 8),
                                     (1024, 4096, 8, 96)])
def test_noalloc_matches_forward_twice(lib, N, K, M, r):
    lora = _layer(N, K, r, seed=N + M)
    g = torch.Generator().manual_seed(M)
    for call in range(2):
        x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
        y_ref = _forward(lib, lora, x, noalloc=False)
        y = _forward(lib, lora, x, noalloc=True)
        assert_matmul_close(y, y_ref, 1)
        assert np.array_equal(y, y_ref), f"call {call}: no-alloc result differs from rq_linear_forward"


def test_noalloc_rejects_requests_beyond_its_scratch(lib):
    """Too large for the built-in scratch: a clear status, nothing launched.
    The buffers are real and sized for the claimed M, so no access could
    leave them even if the check were missing."""
    from rocm_qlora import _native as nat
    N, K, r = 256, 256, 64
    M = 65536
    assert lib.rq_linear_workspace_bytes(M, N, K, r) > SCRATCH_BYTES
    lora = _layer(N, K, r, seed=5)
    w = lora.base_layer.weight_view()
    x = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    y = torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda")
    A = lora.lora_A.detach().bfloat16().contiguous()
    B = lora.lora_B.detach().bfloat16().contiguous()
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.rq_linear_forward_noalloc(*w.args(), x.data_ptr(), nat.BF16, M, None, None, 0, A.data_ptr(),
                                       B.data_ptr(), r, 2.0, y.data_ptr(), st)
    assert rc == RQ_ERR_SCRATCH
    assert b"scratch" in lib.rq_status_string(rc)
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())
