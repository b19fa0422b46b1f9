"""Torch-CPU restatement of the reference's eager QuantLinear+LoRA forward.

TEST / BASELINE INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its
``--impl reference`` arm time this on the host cores as the reference's CPU
implementation of the path.  It performs the same torch operations the
reference performs on the CPU (its own code cannot travel to the GPU box):

* NF4 quantize: per-block absmax, division in the input dtype, nearest
  level by argmin over the fp32 distances, two codes per byte
  (rocm_qlora/quantization/quant_ops.py:80-126);
* NF4 dequantize: code table lookup in fp32, times the block scales
  (rocm_qlora/quantization/quant_ops.py:128-150);
* double-quant first level: c2 (float8_e4m3fnuz) to fp32 times c2_scales
  (rocm_qlora/quantization/double_quant.py:99-122);
* ``F.linear(x, W.to(x.dtype))`` plus ``x @ A.T @ B.T * scaling`` in the
  activation dtype (quant_linear.py:191-197, lora_layer.py:63-70).
"""
import torch
import torch.nn.functional as F

NF4_LEVELS = [
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]


def nf4_quantize(t: torch.Tensor, block_size: int = 64):
    """quantize_int4 (quant_ops.py:80-126): (packed uint8, scales in t's dtype)."""
    flat = t.reshape(-1)
    pad = (-flat.numel()) % block_size
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    blocks = flat.view(-1, block_size)
    scales = blocks.abs().amax(dim=1, keepdim=True).clamp(min=1e-12)
    n = blocks / scales
    table = torch.tensor(NF4_LEVELS, dtype=torch.float32)
    codes = (n.unsqueeze(-1) - table).abs().argmin(dim=-1).to(torch.uint8).reshape(-1)
    packed = codes[0::2] | (codes[1::2] << 4)
    return packed, scales.squeeze()


def nf4_dequantize(packed: torch.Tensor, scales: torch.Tensor, block_size: int = 64) -> torch.Tensor:
    table = torch.tensor(NF4_LEVELS, dtype=torch.float32)
    codes = torch.stack([packed & 0x0F, packed >> 4], dim=1).reshape(-1)
    vals = table[codes.long()].view(-1, block_size)
    return (vals * scales.reshape(-1, 1)).reshape(-1)


def dq_first_level(c2: torch.Tensor, c2_scales: torch.Tensor, nb: int, block2: int = 256) -> torch.Tensor:
    c1 = c2.view(torch.float8_e4m3fnuz).view(-1, block2).to(torch.float32) * c2_scales.reshape(-1, 1)
    return c1.reshape(-1)[:nb]


def loralinear_forward_dq(x, packed, c2, c2_scales, N, K, A, B, scaling):
    """LoRALinear(QuantLinear with double quant).forward in eval mode."""
    c1 = dq_first_level(c2, c2_scales, N * K // 64)
    w = nf4_dequantize(packed, c1)[:N * K].reshape(N, K).to(x.dtype)
    base = F.linear(x, w)
    lora = x @ A.to(x.dtype).T @ B.to(x.dtype).T * scaling
    return base + lora.to(base.dtype)
