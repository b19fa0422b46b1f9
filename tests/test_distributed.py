"""Column-sharded QuantLinear + LoRA: the sharding and collective plumbing.

CPU tests run two `gloo` ranks (spawned processes) with a plain-torch stand-in
for the per-rank layer (the B200 layer needs a GPU), and check the gathered
forward, the all-reduced input and LoRA-A gradients and the local LoRA-B
gradient against the unsharded computation.  The GPU test checks that the
one-rank layer built by ColumnParallelLinear.from_linear is the package's
fused layer.
"""
import os
import socket
import sys

import pytest
import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (ROOT, os.path.join(ROOT, "rocm-qlora_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from rocm_qlora.distributed import ColumnParallelLinear, init_distributed, shard_range  # noqa: E402


@pytest.mark.parametrize("n,world", [(4096, 8), (11008, 8), (28672, 8), (100, 3), (40, 2), (16, 4), (1, 2)])
def test_shard_range_partitions_rows(n, world):
    ranges = [shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 16
    assert all(a % 16 == 0 for a, _ in ranges)


def test_init_distributed_needs_rendezvous(monkeypatch):
    monkeypatch.delenv("MASTER_ADDR", raising=False)
    monkeypatch.delenv("MASTER_PORT", raising=False)
    with pytest.raises(RuntimeError, match="MASTER_ADDR/MASTER_PORT not set"):
        init_distributed(backend="gloo")


class _TorchLoRAShard(nn.Module):
    """Stand-in for one rank's LoRALinear: fp32 torch math over rows of W."""

    def __init__(self, W, A, B, scaling):
        super().__init__()
        self.W = W
        self.lora_A = nn.Parameter(A.clone())
        self.lora_B = nn.Parameter(B.clone())
        self.scaling = scaling

    def forward(self, x):
        return x @ self.W.t() + (x @ self.lora_A.t()) @ self.lora_B.t() * self.scaling


def _rank_main(rank, world, port, N, K, M, r):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    init_distributed(backend="gloo", timeout_minutes=1)
    try:
        g = torch.Generator().manual_seed(11)
        W = torch.randn(N, K, generator=g)
        A = torch.randn(r, K, generator=g)
        B = torch.randn(N, r, generator=g)
        X = torch.randn(M, K, generator=g)
        dY = torch.randn(M, N, generator=g)
        ref = _TorchLoRAShard(W, A, B, 2.0)
        x_ref = X.clone().requires_grad_(True)
        ref(x_ref).backward(dY)

        lo, hi = shard_range(N, world, rank)
        # gather_tokens asks for the fused NVLink gather; without NCCL (gloo)
        # the layer keeps the collective path
        layer = ColumnParallelLinear(_TorchLoRAShard(W[lo:hi], A, B[lo:hi], 2.0), N, gather_tokens=16)
        assert (layer.lo, layer.hi) == (lo, hi) and layer.peer is None
        x = X.clone().requires_grad_(True)
        y = layer(x)
        torch.testing.assert_close(y, ref(X), rtol=1e-5, atol=1e-4)
        y.backward(dY)
        torch.testing.assert_close(x.grad, x_ref.grad, rtol=1e-5, atol=1e-4)
        torch.testing.assert_close(layer.local.lora_A.grad, ref.lora_A.grad, rtol=1e-5, atol=1e-3)
        torch.testing.assert_close(layer.local.lora_B.grad, ref.lora_B.grad[lo:hi], rtol=1e-5, atol=1e-4)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("N", [64, 40])  # 40: uneven shards (16 + 24 rows)
def test_column_parallel_two_gloo_ranks(N):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), N, 32, 5, 4), nprocs=2, join=True)


@pytest.mark.gpu
def test_one_rank_layer_is_the_fused_layer():
    from rocm_qlora import LoRALinear
    torch.manual_seed(0)
    lin = nn.Linear(1024, 512, bias=True, dtype=torch.bfloat16, device="cuda")
    layer = ColumnParallelLinear.from_linear(lin, bits=4, lora_r=8, lora_alpha=16)
    assert layer.world == 1 and isinstance(layer.local, LoRALinear)
    with torch.no_grad():
        layer.local.lora_B.normal_(0, 0.01)
    x = torch.randn(4, 1024, dtype=torch.bfloat16, device="cuda")
    torch.testing.assert_close(layer(x), layer.local(x), rtol=0, atol=0)


# ------------------------------------- sharding an already-quantized layer

def _prequant_layer(N, K, fmt, seed):
    """A QuantLinear (CPU buffers, the reference's layout) built by the
    oracle, as a checkpoint written by the reference would hold it."""
    import numpy as np
    from oracle import oracle as orc
    from rocm_qlora import QuantLinear
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    wb = W.view(torch.int16).numpy().view(np.uint16).reshape(-1)
    bits = 8 if fmt.startswith("int8") else 4
    ql = QuantLinear(K, N, bits=bits, bias=True, block_size=64)
    ql.bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    if fmt == "nf4_dq":
        packed, scales = orc.nf4_quantize(wb, orc.BF16, 64)
        c2, c2s = orc.enable_double_quant(packed, scales, orc.BF16, N * K)
        ql.weight_quant = torch.from_numpy(packed)
        ql.register_buffer("c2", torch.from_numpy(c2).view(torch.float8_e4m3fnuz))
        ql.register_buffer("c2_scales", torch.from_numpy(c2s))
        ql.blocksize_2, ql.use_fp8_c2, ql.use_double_quant = 256, True, True
        ql.weight_scales = torch.empty(0)
    elif fmt == "nf4":
        packed, scales = orc.nf4_quantize(wb, orc.BF16, 64)
        ql.weight_quant = torch.from_numpy(packed)
        ql.weight_scales = torch.from_numpy(scales.view(np.int16)).view(torch.bfloat16)
    elif fmt == "int8_row":
        q, s = orc.int8_quantize_rows(wb.reshape(N, K), orc.BF16)
        ql.weight_quant = torch.from_numpy(q)
        ql.weight_scales = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16)
    return ql


def _dequant(ql):
    import numpy as np
    from oracle import oracle as orc
    from tests.gpu_util import to_bits
    N, K = ql.out_features, ql.in_features
    q = to_bits(ql.weight_quant).reshape(-1)
    if ql.bits == 4 and getattr(ql, "use_double_quant", False):
        return orc.double_dequantize(q, to_bits(ql.c2).reshape(-1), to_bits(ql.c2_scales).reshape(-1),
                                     N * K).reshape(N, K)
    if ql.bits == 4:
        return orc.nf4_dequantize(q, to_bits(ql.weight_scales).reshape(-1), orc.BF16)[:N * K].reshape(N, K)
    return orc.int8_dequantize(q, to_bits(ql.weight_scales).reshape(-1), orc.BF16, rows=N, cols=K).reshape(N, K)


def _prequant_rank(rank, world, port, N, K, fmt, q):
    import numpy as np
    import torch.distributed as dist
    from rocm_qlora import LoRALinear
    from tests.gpu_util import to_bits
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        ql = _prequant_layer(N, K, fmt, seed=N + K)
        lora = LoRALinear(ql, r=8, lora_alpha=16)
        with torch.no_grad():
            lora.lora_B.normal_(0, 0.01, generator=torch.Generator().manual_seed(3))
        cp = ColumnParallelLinear.from_quant_linear(lora, gather_tokens=0)
        loc = cp.local.base_layer
        lo, hi = cp.lo, cp.hi
        # the shard dequantizes to exactly the full layer's rows
        full = _dequant(ql)
        same = np.array_equal(_dequant(loc).view(np.uint32), full[lo:hi].view(np.uint32))
        # and its bytes are slices of the full layer's
        b0 = lo * K // 64
        sl = to_bits(loc.weight_quant).reshape(-1)
        if fmt == "int8_row":
            ok_bytes = np.array_equal(sl, to_bits(ql.weight_quant)[lo:hi].reshape(-1))
        else:
            per = 2 if ql.bits == 4 else 1
            ok_bytes = np.array_equal(sl, to_bits(ql.weight_quant).reshape(-1)[b0 * 64 // per:b0 * 64 // per + sl.size])
        if fmt == "nf4_dq":
            ok_bytes = ok_bytes and b0 % 256 == 0 and np.array_equal(
                to_bits(loc.c2).reshape(-1), to_bits(ql.c2).reshape(-1)[b0:b0 + to_bits(loc.c2).size])
        ok_lora = torch.equal(cp.local.lora_B, lora.lora_B[lo:hi]) and torch.equal(cp.local.lora_A, lora.lora_A)
        sizes = [None] * world
        dist.all_gather_object(sizes, (lo, hi))
        q.put((rank, bool(same), bool(ok_bytes), bool(ok_lora), sizes))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), False, False, None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("N,K,fmt", [(1000, 11008, "nf4_dq"), (600, 1088, "nf4_dq"), (300, 4096, "nf4"),
                                     (257, 2048, "int8_row")])
def test_from_quant_linear_three_ranks(N, K, fmt):
    """Sharding a reference-quantized layer over three gloo ranks: every
    shard's codes, c2 bytes and c2_scales are slices of the full layer's, they
    dequantize to the same values as the full layer's rows (second-level
    groups never straddle a shard boundary: K = 11008 has 172 blocks a row,
    so shards start at multiples of 64 rows), and the shards tile the rows."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_prequant_rank, args=(r, 3, port, N, K, fmt, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, same, ok_bytes, ok_lora, sizes in res:
        assert same is True, f"rank {rank}: {same}"
        assert ok_bytes and ok_lora, f"rank {rank}"
    sizes = res[0][4]
    assert sizes[0][0] == 0 and sizes[-1][1] == N
    assert all(a[1] == b[0] for a, b in zip(sizes, sizes[1:]))
