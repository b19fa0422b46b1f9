"""Two-rank GPU tests of the column-sharded layer with the fused gather:
the decode GEMV writes each rank's output features into every rank's full
output over NVLink (rocm_qlora.distributed.peer_gather).

The gathered output must equal, bit for bit, (a) the NCCL all-gather path of
the same sharded layer and (b) the unsharded layer on one GPU: with K a
multiple of 64 the shards quantize to the same codes and scales as the
full weight's rows, and the GEMV's per-row reduction order does not depend
on the shard.  Needs two GPUs (one process per GPU, NCCL over 127.0.0.1);
skipped otherwise."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [
    # full out_features, K, M, LoRA r, bias
    (4096, 4096, 1, 16, False),
    (22016, 4096, 16, 16, False),   # 2 x 11008
    (1000, 1024, 4, 0, True),       # uneven shards (496 / 504 rows), no adapter
    (4096, 11008, 8, 16, True),     # K not a multiple of 256
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "rocm-qlora_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    import torch.nn as nn
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    ok = False
    try:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from rocm_qlora import LoRALinear, QuantLinear
        from rocm_qlora import _native as nat
        from rocm_qlora.distributed import ColumnParallelLinear
        import ctypes
        msgs = []
        for (Nt, K, M, r, bias) in CASES:
            g = torch.Generator().manual_seed(Nt + K + M + r)
            W = (torch.randn(Nt, K, generator=g) * 0.02).to(torch.bfloat16)
            bvec = (torch.randn(Nt, generator=g) * 0.1).to(torch.bfloat16) if bias else None
            A = (torch.rand(max(r, 1), K, generator=g) * 2 - 1) / K ** 0.5
            B = torch.randn(Nt, max(r, 1), generator=g) * 0.01
            X = torch.randn(M, K, generator=g).to(torch.bfloat16)
            lin = nn.Linear(K, Nt, bias=bias, dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                lin.weight.copy_(W.to(dev))
                if bias:
                    lin.bias.copy_(bvec.to(dev))
            cp = ColumnParallelLinear.from_linear(lin, bits=4, double_quant=True, lora_r=r, lora_alpha=2 * max(r, 1),
                                                  gather_tokens=16)
            assert cp.peer is not None
            if r:
                with torch.no_grad():
                    cp.local.lora_A.copy_(A.to(dev))
                    cp.local.lora_B.copy_(B[cp.lo:cp.hi].to(dev))
            cp.eval()
            x = X.to(dev)
            with torch.no_grad():
                y_fused = cp(x).clone()
                assert nat.lib().rq_last_path() == 1  # the decode GEMV ran
                peer, cp.peer = cp.peer, None
                y_nccl = cp(x)
                cp.peer = peer
            assert not peer.error(), "a rank gave up waiting for a peer"
            c = ctypes.c_uint(0)
            assert nat.lib().rq_take_kernel_timeouts(ctypes.byref(c)) == 0 and c.value == 0
            assert torch.equal(y_fused, y_nccl), f"fused != NCCL for {(Nt, K, M, r, bias)}"
            # the unsharded layer on this GPU
            ql = QuantLinear.from_linear(lin, bits=4)
            ql.enable_double_quant()
            full = LoRALinear(ql, r=r, lora_alpha=2 * r).to(dev).eval() if r else ql
            if r:
                with torch.no_grad():
                    full.lora_A.copy_(A.to(dev))
                    full.lora_B.copy_(B.to(dev))
            with torch.no_grad():
                y_full = full(x)
            assert torch.equal(y_fused, y_full), f"fused != unsharded for {(Nt, K, M, r, bias)}"
            cp.close()
            msgs.append(f"{(Nt, K, M, r, bias)} ok")
        ok = True
        q.put((rank, "ok", msgs))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), []))
    finally:
        if dist.is_initialized():
            if ok:
                dist.barrier()
            dist.destroy_process_group()


def _setup(rank, world, port):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "rocm-qlora_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    return dev


def _sharded(dev, Nt, K, r, seed):
    import torch.nn as nn
    from rocm_qlora.distributed import ColumnParallelLinear
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(Nt, K, generator=g) * 0.02).to(torch.bfloat16)
    A = (torch.rand(r, K, generator=g) * 2 - 1) / K ** 0.5
    B = torch.randn(Nt, r, generator=g) * 0.01
    lin = nn.Linear(K, Nt, bias=False, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        lin.weight.copy_(W.to(dev))
    cp = ColumnParallelLinear.from_linear(lin, bits=4, double_quant=True, lora_r=r, lora_alpha=2 * r,
                                          gather_tokens=16)
    with torch.no_grad():
        cp.local.lora_A.copy_(A.to(dev))
        cp.local.lora_B.copy_(B[cp.lo:cp.hi].to(dev))
    return cp.eval()


def _nccl(cp, x):
    peer, cp.peer = cp.peer, None
    try:
        with torch.no_grad():
            return cp(x).clone()
    finally:
        cp.peer = peer


def _worker_slow_reader(rank: int, world: int, port: int, q) -> None:
    """Back-to-back fused calls of one layer while rank 1 reads the first
    result late (a 50 ms device sleep before its copy): rank 0's second call
    must not overwrite rank 1's copy of the first result before rank 1 has
    read it (rank 0 stores only after rank 1 entered the second call)."""
    import torch.distributed as dist
    ok = False
    try:
        dev = _setup(rank, world, port)
        cp = _sharded(dev, 4096, 4096, 16, seed=11)
        g = torch.Generator().manual_seed(12)
        xa = torch.randn(4, 4096, generator=g).to(torch.bfloat16).to(dev)
        xb = torch.randn(4, 4096, generator=g).to(torch.bfloat16).to(dev)
        ya_ref, yb_ref = _nccl(cp, xa), _nccl(cp, xb)
        torch.cuda.synchronize()
        dist.barrier()
        with torch.no_grad():
            ya = cp(xa)
            if rank == 1:
                torch.cuda._sleep(100_000_000)  # ~50 ms at 1.9 GHz before this rank reads its result
            ya_read = ya.clone()
            yb = cp(xb).clone()
        torch.cuda.synchronize()
        assert not cp.peer.error(), "a rank gave up waiting"
        assert torch.equal(ya_read, ya_ref), f"rank {rank}: first result overwritten before it was read"
        assert torch.equal(yb, yb_ref), f"rank {rank}: second result differs from NCCL"
        cp.close()
        ok = True
        q.put((rank, "ok", ["slow reader ok"]))
    except Exception as e:
        q.put((rank, repr(e), []))
    finally:
        if dist.is_initialized():
            if ok:
                dist.barrier()
            dist.destroy_process_group()


def _worker_missing_rank(rank: int, world: int, port: int, q) -> None:
    """Rank 1 skips one fused call (a host-side fault: the call is never
    issued).  Rank 0's kernel gives up its bounded waits (about 2 s each),
    returns with the error flag raised and counts the timeouts; nothing
    hangs and both ranks close cleanly."""
    import ctypes
    import time
    import torch.distributed as dist
    from rocm_qlora import _native as nat
    ok = False
    try:
        dev = _setup(rank, world, port)
        cp = _sharded(dev, 2048, 1024, 16, seed=21)
        x = torch.randn(2, 1024, generator=torch.Generator().manual_seed(22)).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            cp(x)  # one good call on both ranks
        torch.cuda.synchronize()
        assert not cp.peer.error()
        dist.barrier()
        t0 = time.perf_counter()
        if rank == 0:
            with torch.no_grad():
                cp(x)  # rank 1 never makes this call
            torch.cuda.synchronize()
            waited = time.perf_counter() - t0
            c = ctypes.c_uint(0)
            assert nat.lib().rq_take_kernel_timeouts(ctypes.byref(c)) == 0
            assert cp.peer.error(), "the missing rank was not reported"
            assert c.value >= 1, "no bounded wait counted a timeout"
            assert waited < 30.0, f"the timed-out call took {waited:.1f} s"
        dist.barrier()
        cp.close()
        ok = True
        q.put((rank, "ok", ["missing rank reported"]))
    except Exception as e:
        q.put((rank, repr(e), []))
    finally:
        if dist.is_initialized():
            if ok:
                dist.barrier()
            dist.destroy_process_group()


def _worker_prequantized(rank: int, world: int, port: int, q) -> None:
    """A layer quantized whole (as a checkpoint holds it) and sharded with
    ColumnParallelLinear.from_quant_linear: the fused decode output equals
    the unsharded layer's bit for bit, also when K = 11008 puts second-level
    groups across rows (shards start at multiples of 64 rows)."""
    import torch.distributed as dist
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.distributed import ColumnParallelLinear
    ok = False
    try:
        dev = _setup(rank, world, port)
        msgs = []
        for (N, K, M) in ((2048, 11008, 16), (1000, 4096, 1)):
            g = torch.Generator().manual_seed(N + K)
            lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                lin.weight.copy_((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev))
            ql = QuantLinear.from_linear(lin, bits=4)
            ql.enable_double_quant()
            full = LoRALinear(ql, r=16, lora_alpha=32).to(dev).eval()
            with torch.no_grad():
                full.lora_A.copy_(((torch.rand(16, K, generator=g) * 2 - 1) / K ** 0.5).to(dev))
                full.lora_B.copy_((torch.randn(N, 16, generator=g) * 0.01).to(dev))
            cp = ColumnParallelLinear.from_quant_linear(full, gather_tokens=16).eval()
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
            with torch.no_grad():
                y = cp(x).clone()
                y_full = full(x)
            assert not cp.peer.error()
            assert torch.equal(y, y_full), f"sharded != unsharded for {(N, K, M)}"
            cp.close()
            msgs.append(f"{(N, K, M)} ok")
        ok = True
        q.put((rank, "ok", msgs))
    except Exception as e:
        q.put((rank, repr(e), []))
    finally:
        if dist.is_initialized():
            if ok:
                dist.barrier()
            dist.destroy_process_group()


def _run_two(target, n_msgs):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    for _ in procs:
        results.append(q.get(timeout=600))
    for p in procs:
        p.join(timeout=120)
    for rank, status, msgs in results:
        assert status == "ok", f"rank {rank}: {status}"
        assert len(msgs) == n_msgs


TWO_GPUS = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs two GPUs")


@TWO_GPUS
def test_fused_gather_two_ranks():
    _run_two(_worker, len(CASES))


@TWO_GPUS
def test_fused_gather_slow_reader():
    _run_two(_worker_slow_reader, 1)


@TWO_GPUS
def test_fused_gather_missing_rank_times_out():
    _run_two(_worker_missing_rank, 1)


@TWO_GPUS
def test_prequantized_layer_sharded_two_ranks():
    _run_two(_worker_prequantized, 2)
