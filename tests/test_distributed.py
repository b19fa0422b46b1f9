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
