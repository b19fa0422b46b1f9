"""Node-wide output buffers for column-sharded layers (the fused gather).

A column-sharded layer computes its output features [lo, hi) on every rank;
the full output Y[M, N] is the concatenation over the ranks.  Instead of a
separate collective after the layer, the decode kernel writes its shard
straight into every rank's copy of Y over NVLink (peer stores) and the ranks
meet at the end of the kernel (a flag per rank, bounded wait).  This module
owns the memory that makes that possible:

  * Y [max_tokens, N] in the activation dtype, one per rank, mapped into
    every other rank's process (CUDA IPC, same node);
  * a flag array of 2 x `world` uint32 per rank, also mapped everywhere (the
    epoch each rank finished, and the epoch each rank entered: a rank writes
    into the others' Y only after all of them entered the call, so a result
    that a slower rank is still reading is never overwritten);
  * 4 uint32 of control state per rank (arrival counter, epoch, error).

Handles travel once through ``all_gather_object`` of the process group.
Construction and ``close`` are collective: every rank of the group calls
them in the same order.  The result of a call lives in ``output(M)`` until
the next gathering call of the same layer (the caller consumes it first).
"""
import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from rocm_qlora import _native as nat


class _DeviceArray:
    """A raw device allocation seen by torch through the CUDA array
    interface (no copy; the memory belongs to the PeerGather)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_TYPESTR = {torch.bfloat16: ("<i2", 2), torch.float16: ("<f2", 2)}


class PeerGather:
    """The gathered output of one column-sharded layer on this rank.

    ``col`` is the first output feature of this rank's shard and
    ``out_features`` the full width N.  ``descriptor`` is the
    ``_native.RqGather`` handed to ``rq_linear_forward_gather``."""

    def __init__(self, group, max_tokens: int, out_features: int, col: int, dtype: torch.dtype,
                 device: torch.device):
        if dtype not in _TYPESTR:
            raise TypeError(f"the fused gather writes bf16 or f16 outputs, not {dtype}")
        if max_tokens < 1:
            raise ValueError("max_tokens must be positive")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.out_features, self.col = max_tokens, out_features, col
        self.dtype, self.device = dtype, torch.device(device)
        L = nat.lib()
        typestr, esz = _TYPESTR[dtype]
        self._own: List[int] = []
        self._opened: List[int] = []
        # Every rank takes part in both exchanges whatever happens locally,
        # and all ranks raise together if any rank failed: the group's
        # collectives stay matched.
        with torch.cuda.device(self.device):
            handles, err = None, None
            try:
                out = self._alloc(L, max_tokens * out_features * esz)
                flags = self._alloc(L, 8 * self.world)  # finished and entered epochs per rank
                self._ctrl = self._alloc(L, 16)
                handles = (self._handle(L, out), self._handle(L, flags))
            except Exception as e:
                err = e
            every = [None] * self.world
            dist.all_gather_object(every, handles, group=group)
            outs, fl = [], []
            if err is None and all(h is not None for h in every):
                try:
                    for q, (ho, hf) in enumerate(every):
                        if q == self.rank:
                            outs.append(out)
                            fl.append(flags)
                        else:
                            outs.append(self._open(L, ho))
                            fl.append(self._open(L, hf))
                except Exception as e:
                    err = e
            else:
                err = err or RuntimeError("another rank could not allocate its shared buffers")
            verdict = [None] * self.world
            dist.all_gather_object(verdict, err is None, group=group)
            if not all(verdict):
                self._release_local(L)
                raise RuntimeError(f"fused gather unavailable on this node: {err!r}" if err is not None
                                   else "fused gather unavailable: another rank failed to map the buffers")
            self._outs_dev = torch.tensor(outs, dtype=torch.int64, device=self.device)
            self._flags_dev = torch.tensor(fl, dtype=torch.int64, device=self.device)
            self.y = torch.as_tensor(_DeviceArray(out, (max_tokens, out_features), typestr),
                                     device=self.device).view(dtype)
            self._ctrl_view = torch.as_tensor(_DeviceArray(self._ctrl, (4,), "<i4"), device=self.device)
        self.descriptor = nat.RqGather(self._outs_dev.data_ptr(), self._flags_dev.data_ptr(), flags, self._ctrl,
                                       out_features, col, self.world, self.rank)

    @staticmethod
    def _alloc_raw(L, nbytes: int) -> int:
        p = ctypes.c_void_p()
        nat.check(L.rq_peer_alloc(nbytes, ctypes.byref(p)), "rq_peer_alloc")
        return p.value

    def _alloc(self, L, nbytes: int) -> int:
        p = self._alloc_raw(L, nbytes)
        self._own.append(p)
        return p

    @staticmethod
    def _handle(L, ptr: int) -> bytes:
        buf = ctypes.create_string_buffer(64)
        nat.check(L.rq_peer_handle(ptr, buf), "rq_peer_handle")
        return buf.raw

    def _open(self, L, handle: bytes) -> int:
        p = ctypes.c_void_p()
        nat.check(L.rq_peer_open(handle, ctypes.byref(p)), "rq_peer_open")
        self._opened.append(p.value)
        return p.value

    def _release_local(self, L) -> None:
        for p in self._opened:
            L.rq_peer_close(p)
        for p in self._own:
            L.rq_peer_free(p)
        self._own, self._opened = None, []

    def output(self, M: int) -> torch.Tensor:
        """Y[:M] of the last gathering call (a view of the shared buffer)."""
        return self.y[:M]

    def error(self) -> bool:
        """True if a call gave up waiting for a peer (reads the device flag)."""
        return bool(self._ctrl_view[2].item())

    def close(self) -> None:
        """Collective: unmap the peers' memory and free this rank's."""
        if self._own is None:
            return
        L = nat.lib()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                nat.check(L.rq_peer_close(p), "rq_peer_close")
            dist.barrier(group=self.group)  # nobody maps this rank's memory any more
            for p in self._own:
                nat.check(L.rq_peer_free(p), "rq_peer_free")
        self._own, self._opened = None, []
        self.y = None


def gather_eligible(x2d: torch.Tensor, local, max_tokens: int) -> bool:
    """The rank-independent part of the fused path's conditions: a decode
    batch (M <= 16, within the buffers), bf16/f16 activations, a 4-bit
    QuantLinear base on the fused path (no merged weight), no active LoRA
    dropout and no autograd graph to record.  Every rank of a call sees the
    same answer."""
    from rocm_qlora.lora.lora_layer import LoRALinear
    from rocm_qlora.quantization.quant_linear import QuantLinear
    lora = isinstance(local, LoRALinear)
    base = local.base_layer if lora else local
    if not isinstance(base, QuantLinear) or base.bits != 4 or (base.merged_mode and base.merged_fp16_weight is not None):
        return False
    if lora and (local.merged or (local.training and isinstance(local.lora_dropout, torch.nn.Dropout)
                                  and local.lora_dropout.p > 0)):
        return False
    if torch.is_grad_enabled() and (x2d.requires_grad or any(p.requires_grad for p in local.parameters())):
        return False
    M = x2d.shape[0]
    return 1 <= M <= min(16, max_tokens) and x2d.dtype in _TYPESTR and x2d.is_cuda
