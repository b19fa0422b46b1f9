"""Column-sharded QuantLinear (+ LoRA) across the GPUs of one node.

The quantized weight W [N, K] is split by output features into contiguous
row ranges, 16 rows apiece where possible (blocks stay whole: with K % 64
== 0 a 64-block never crosses a row).  Rank i holds rows [lo_i, hi_i) of W,
of the bias and of LoRA B; LoRA A [r, K] is replicated.

  forward    Y_i = layer_i(X);  Y = all-gather of the Y_i over the features
  backward   dX  = sum over ranks of dX_i  (all-reduce)
             dA  = sum over ranks of dA_i  (all-reduce; A is replicated)
             dB_i, dbias_i stay local

The collectives are NCCL over NVLink (torch.distributed); the per-rank
layer is the fused B200 QuantLinear / LoRALinear of this package.  With
``gather_tokens > 0`` the decode forward (M <= 16, no autograd) skips the
all-gather: the GEMV writes its shard into every rank's output over NVLink
and the ranks meet at the end of the kernel (``peer_gather.PeerGather``).
"""
import math
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from rocm_qlora import _native as nat
from rocm_qlora.distributed.peer_gather import PeerGather, gather_eligible
from rocm_qlora.lora.lora_layer import LoRALinear
from rocm_qlora.quantization import layer_ops
from rocm_qlora.quantization.quant_linear import QuantLinear


def shard_range(n: int, world: int, rank: int, granule: int = 16) -> Tuple[int, int]:
    """Rows [lo, hi) of `rank` when `n` rows are split over `world` ranks in
    units of `granule` rows (the last unit may be short); shard sizes differ
    by at most one unit."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    units = -(-n // granule)
    lo = units * rank // world * granule
    hi = units * (rank + 1) // world * granule
    return min(lo, n), min(hi, n)


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


class _ReduceGradient(torch.autograd.Function):
    """Identity forward; the gradient is summed over the group (the input is
    replicated, every rank's shard contributes to its gradient)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _GatherFeatures(torch.autograd.Function):
    """All-gather of the ranks' output features along the last dimension;
    the gradient of each rank is its own slice."""

    @staticmethod
    def forward(ctx, y, group, sizes: List[int], rank: int):
        ctx.lo = sum(sizes[:rank])
        ctx.n = sizes[rank]
        nmax = max(sizes)
        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1])
        if y2.shape[1] < nmax:  # uneven shards: pad to the largest
            y2 = torch.nn.functional.pad(y2, (0, nmax - y2.shape[1]))
        buf = torch.empty((len(sizes), y2.shape[0], nmax), dtype=y.dtype, device=y.device)
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(buf, y2.contiguous(), group=group)
        else:  # gloo has no single-buffer all-gather
            dist.all_gather(list(buf.unbind(0)), y2.contiguous(), group=group)
        out = torch.cat([buf[i, :, :sizes[i]] for i in range(len(sizes))], dim=1)
        return out.reshape(*lead, sum(sizes))

    @staticmethod
    def backward(ctx, g):
        return g[..., ctx.lo:ctx.lo + ctx.n].contiguous(), None, None, None


class ColumnParallelLinear(nn.Module):
    """One rank's shard of a column-sharded layer.

    `local` computes this rank's output features (a QuantLinear or
    LoRALinear over rows [lo, hi) of the full weight); `out_features` is the
    full width.  A LoRA A parameter of `local` is treated as replicated: its
    gradient is all-reduced during backward.
    """

    def __init__(self, local: nn.Module, out_features: int, group=None, granule: int = 16, gather_tokens: int = 0,
                 gather_dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.local = local
        self.group = group
        self.out_features = out_features
        self.world, self.rank = _world(group)
        self.sizes = [b - a for a, b in (shard_range(out_features, self.world, i, granule) for i in range(self.world))]
        self.lo, self.hi = shard_range(out_features, self.world, self.rank, granule)
        self.peer: Optional[PeerGather] = None
        if gather_tokens > 0 and self.world > 1 and dist.get_backend(group) == "nccl":
            dev = next(local.buffers()).device
            self.peer = PeerGather(group, gather_tokens, out_features, self.lo, gather_dtype, dev)
        lora_a = getattr(local, "lora_A", None)
        if self.world > 1 and isinstance(lora_a, torch.Tensor) and lora_a.requires_grad:
            lora_a.register_hook(self._sum_over_ranks)

    def _sum_over_ranks(self, g: torch.Tensor) -> torch.Tensor:
        g = g.contiguous().clone()
        dist.all_reduce(g, group=self.group)
        return g

    def _forward_fused(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        """The gathered output through the fused kernel, or None when this
        call has no fused form (decided identically on every rank)."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if self.peer is None or x2.dtype != self.peer.dtype or not gather_eligible(x2, self.local, self.peer.max_tokens):
            return None
        x2 = x2.contiguous()
        if isinstance(self.local, LoRALinear):
            base, dt = self.local.base_layer, x2.dtype
            A, B = layer_ops.cast_param(self.local.lora_A, dt), layer_ops.cast_param(self.local.lora_B, dt)
            s = self.local.scaling
        else:
            base, A, B, s = self.local, None, None, 1.0
        bias = base.bias.to(x2.dtype).contiguous() if base.bias is not None else None
        rc = layer_ops.forward_gather(base.weight_view(), x2, bias, A, B, s, self.peer.descriptor)
        if rc != nat.RQ_OK:
            # nothing was launched on this rank, but the others may have: a
            # hang must not follow, so this is an error, not a fallback
            raise RuntimeError("rq_linear_forward_gather refused a call the ranks agreed to fuse")
        return self.peer.output(x2.shape[0]).view(*lead, self.out_features)

    def close(self) -> None:
        """Collective: release the fused-gather buffers (every rank calls it)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return self.local(x)
        y = self._forward_fused(x)
        if y is not None:
            return y
        if torch.is_grad_enabled() and x.requires_grad:
            x = _ReduceGradient.apply(x, self.group)
        y = self.local(x)
        return _GatherFeatures.apply(y, self.group, self.sizes, self.rank)

    @classmethod
    def from_linear(cls, linear: nn.Linear, bits: int = 4, double_quant: bool = True, lora_r: int = 0,
                    lora_alpha: int = 16, lora_dropout: float = 0.0, group=None,
                    granule: int = 16, gather_tokens: int = 0) -> "ColumnParallelLinear":
        """Quantizes this rank's rows of `linear` (every rank passes the same
        full layer) and wraps them, with LoRA adapters when lora_r > 0 (A
        broadcast from rank 0 so all ranks hold the same replica; B starts at
        zero as in LoRALinear)."""
        world, rank = _world(group)
        lo, hi = shard_range(linear.out_features, world, rank, granule)
        shard = nn.Linear(linear.in_features, hi - lo, bias=linear.bias is not None,
                          dtype=linear.weight.dtype, device=linear.weight.device)
        with torch.no_grad():
            shard.weight.copy_(linear.weight[lo:hi])
            if linear.bias is not None:
                shard.bias.copy_(linear.bias[lo:hi])
        local: nn.Module = QuantLinear.from_linear(shard, bits=bits)
        if double_quant and bits == 4:
            local.enable_double_quant()
        if lora_r > 0:
            local = LoRALinear(local, r=lora_r, lora_alpha=lora_alpha, lora_dropout=lora_dropout).to(
                linear.weight.device)
            if world > 1:
                with torch.no_grad():
                    dist.broadcast(local.lora_A.data, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        return cls(local, linear.out_features, group=group, granule=granule, gather_tokens=gather_tokens,
                   gather_dtype=linear.weight.dtype if linear.weight.dtype in (torch.bfloat16, torch.float16)
                   else torch.bfloat16)

    @classmethod
    def from_quant_linear(cls, layer: nn.Module, group=None, granule: int = 16,
                          gather_tokens: int = 0) -> "ColumnParallelLinear":
        """Shards an already-quantized layer (a QuantLinear, or a LoRALinear
        over one, holding the full weight on every rank -- e.g. loaded from a
        checkpoint written by the reference) without re-quantizing: each rank
        keeps its rows' codes and scales byte for byte.

        Shard boundaries are rows r with r*K a multiple of the block size (no
        block spans two shards) and, with double-quantized scales, r*K/64 a
        multiple of the 256-block second-level group, so each shard's c2
        bytes and c2_scales are a contiguous slice of the full layer's and
        dequantize to exactly the same values (double_quant.py:46-97 of the
        reference groups the flat block list in 256s).  LoRA B is sliced by
        rows, LoRA A is kept whole (replicated)."""
        world, rank = _world(group)
        lora = layer if isinstance(layer, LoRALinear) else None
        ql = lora.base_layer if lora is not None else layer
        if not isinstance(ql, QuantLinear):
            raise TypeError("from_quant_linear takes a QuantLinear or a LoRALinear over one")
        N, K, bs = ql.out_features, ql.in_features, ql.block_size
        dq = ql.bits == 4 and getattr(ql, "use_double_quant", False)
        per_row = ql.bits == 8 and ql.weight_quant.dim() == 2 and ql.weight_scales.numel() == N
        unit = granule
        if not per_row:
            unit = math.lcm(unit, bs // math.gcd(K, bs))  # whole blocks per shard
        if dq:
            bs2 = getattr(ql, "blocksize_2", 256)
            unit = math.lcm(unit, (bs * bs2) // math.gcd(K, bs * bs2))  # whole second-level groups
        lo, hi = shard_range(N, world, rank, unit)
        local = QuantLinear(K, hi - lo, bits=ql.bits, bias=ql.bias is not None, block_size=bs)
        local.original_shape = (hi - lo, K)
        if per_row:
            local.weight_quant = ql.weight_quant[lo:hi].clone()
            local.weight_scales = ql.weight_scales.reshape(-1)[lo:hi].clone()
        else:
            per_byte = 2 if ql.bits == 4 else 1
            b0, b1 = lo * K // bs, -(-(hi * K) // bs)
            local.weight_quant = ql.weight_quant.reshape(-1)[b0 * bs // per_byte:b1 * bs // per_byte].clone()
            if dq:
                g0, g1 = b0 // bs2, -(-b1 // bs2)
                local.register_buffer("c2", ql.c2.reshape(-1)[g0 * bs2:g1 * bs2].clone())
                local.register_buffer("c2_scales", ql.c2_scales.reshape(-1)[g0:g1].clone())
                local.blocksize_2 = bs2
                local.use_fp8_c2 = getattr(ql, "use_fp8_c2", True)
                local.use_double_quant = True
                local.weight_scales = ql.weight_scales.new_empty(0)
            else:
                local.weight_scales = ql.weight_scales.reshape(-1)[b0:b1].clone()
        if ql.bias is not None:
            local.bias = ql.bias[lo:hi].clone()
        local.use_triton_kernel = ql.use_triton_kernel
        shard: nn.Module = local
        if lora is not None:
            shard = LoRALinear(local, r=lora.r, lora_alpha=lora.lora_alpha,
                               lora_dropout=lora.lora_dropout.p if isinstance(lora.lora_dropout, nn.Dropout) else 0.0)
            shard = shard.to(lora.lora_A.device)
            with torch.no_grad():
                shard.lora_A.copy_(lora.lora_A)
                shard.lora_B.copy_(lora.lora_B[lo:hi])
            shard.train(lora.training)
        dtype = ql.bias.dtype if ql.bias is not None else torch.bfloat16
        return cls(shard, N, group=group, granule=unit, gather_tokens=gather_tokens,
                   gather_dtype=dtype if dtype in (torch.bfloat16, torch.float16) else torch.bfloat16)
