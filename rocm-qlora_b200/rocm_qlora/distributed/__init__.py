"""Multi-GPU support: process-group plumbing (the reference's launch
utilities) and the column-sharded QuantLinear + LoRA layer."""
from rocm_qlora.distributed.launch_utils import (
    barrier, cleanup_distributed, get_distributed_info, init_distributed, is_main_process, print_on_main,
    setup_device,
)
from rocm_qlora.distributed.column_parallel import ColumnParallelLinear, shard_range

__all__ = [
    "init_distributed", "setup_device", "cleanup_distributed", "is_main_process", "print_on_main", "barrier",
    "get_distributed_info", "ColumnParallelLinear", "shard_range",
]
