"""Process-group plumbing for multi-GPU runs (one process per GPU, NCCL).

Same names and behaviour as the reference's
rocm_qlora/distributed/launch_utils.py:17-81: torchrun sets RANK /
LOCAL_RANK / WORLD_SIZE / MASTER_*; ``init_distributed`` refuses to start
without a rendezvous address, with the reference's message.  On B200 the
"nccl" backend is NCCL over NVLink 5 / NVSwitch.
"""
import os
from datetime import timedelta
from typing import Any, Dict, Tuple

import torch
import torch.distributed as dist


def init_distributed(backend: str = "nccl", timeout_minutes: int = 30) -> Tuple[int, int, int]:
    """Joins the process group; returns (rank, local_rank, world_size)."""
    if "MASTER_ADDR" not in os.environ or "MASTER_PORT" not in os.environ:
        raise RuntimeError("MASTER_ADDR/MASTER_PORT not set. "
                           "Please launch with: torchrun --nproc_per_node=N script.py")
    rank = int(os.environ.get("RANK", 0))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    world_size = int(os.environ.get("WORLD_SIZE", 1))
    dist.init_process_group(backend=backend, timeout=timedelta(minutes=timeout_minutes))
    return rank, local_rank, world_size


def setup_device(local_rank: int) -> torch.device:
    """Selects and returns this process's GPU (the CPU device when the host
    has none: device selection only, every kernel of this package needs a
    GPU)."""
    if not torch.cuda.is_available():
        return torch.device("cpu")
    torch.cuda.set_device(local_rank)
    return torch.device(f"cuda:{local_rank}")


def cleanup_distributed() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def is_main_process(rank: int) -> bool:
    return rank == 0


def print_on_main(message: str, rank: int) -> None:
    if rank == 0:
        print(message)


def barrier(rank: int) -> None:
    if dist.is_initialized():
        dist.barrier()


def get_distributed_info() -> Dict[str, Any]:
    return {
        "rank": int(os.environ.get("RANK", -1)),
        "local_rank": int(os.environ.get("LOCAL_RANK", -1)),
        "world_size": int(os.environ.get("WORLD_SIZE", -1)),
        "backend": dist.get_backend() if dist.is_initialized() else "none",
        "nccl_available": torch.cuda.is_available() and dist.is_nccl_available(),
    }
