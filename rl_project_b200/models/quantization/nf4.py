"""4-bit NormalFloat (NF4) block quantisation: block 64, per-block absmax,
two indices per byte, high nibble first (``src/forgeline/models/quantization/nf4.py``).

The 16 NF4 levels are the QLoRA paper's normal-quantile table (Dettmers et
al., 2023), the same data the reference ships.  On CUDA, ``NF4Linear``
dequantises in the sm_100a kernel csrc/nf4.cu straight to bf16 in one pass
(the reference dequantises through fp32 index tensors on every forward); with
``RLB_NF4_GEMM=1`` the forward and input gradient instead run csrc/nf4_gemm.cu,
which expands the weight tile by tile inside the tcgen05 GEMM (tested on B200
against an fp32 matmul of the dequantised weight).
"""

from __future__ import annotations

import os
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import QuantizationError

NF4_TABLE = torch.tensor([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
], dtype=torch.float32)
NF4_BLOCK_SIZE = 64


def quantize_nf4(tensor: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Size]:
    if tensor.numel() == 0:
        raise QuantizationError("cannot quantize an empty tensor")
    flat = tensor.detach().reshape(-1).float().cpu()
    pad = (-flat.numel()) % NF4_BLOCK_SIZE
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    blocks = flat.view(-1, NF4_BLOCK_SIZE)
    absmax = blocks.abs().amax(1).clamp(min=1e-8)
    normed = blocks / absmax[:, None]
    # nearest level: midpoints between sorted levels partition [-1, 1]
    mids = (NF4_TABLE[1:] + NF4_TABLE[:-1]) / 2
    idx = torch.bucketize(normed.reshape(-1), mids)
    packed = ((idx[0::2] << 4) | idx[1::2]).to(torch.uint8)
    return packed, absmax, tensor.shape


def dequantize_nf4(packed: torch.Tensor, absmax: torch.Tensor, shape: torch.Size,
                   dtype: torch.dtype = torch.float32) -> torch.Tensor:
    n = 1
    for s in shape:
        n *= int(s)
    if packed.is_cuda:
        from rl_project_b200.ops._ext import native

        out = native().nf4_dequant(packed, absmax.float().contiguous(), NF4_TABLE.to(packed.device), n,
                                   NF4_BLOCK_SIZE, dtype == torch.bfloat16)
        return out.view(shape).to(dtype)
    idx = torch.stack([(packed >> 4).long(), (packed & 0x0F).long()], -1).reshape(-1)
    vals = NF4_TABLE[idx].view(-1, NF4_BLOCK_SIZE) * absmax.float().cpu()[:, None]
    return vals.reshape(-1)[:n].view(shape).to(dtype)


_NF4_GEMM = os.environ.get("RLB_NF4_GEMM", "0") == "1"
_STATUS: dict = {}


def _status(device: torch.device) -> torch.Tensor:
    if device.index not in _STATUS:
        _STATUS[device.index] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STATUS[device.index]


class _NF4Matmul(torch.autograd.Function):
    """``x @ W^T`` with the NF4 weight expanded inside the tcgen05 GEMM (csrc/nf4_gemm.cu); the backward
    is the same kernel's ``dy @ W`` (the quantised base weight is frozen: no weight gradient)."""

    @staticmethod
    def forward(ctx, x2, lin):
        from rl_project_b200.ops._ext import native

        ctx.lin = lin
        N, K = lin.weight_shape
        return native().nf4_gemm(x2, lin.weight_packed, lin.weight_absmax.float(), lin._table(x2.device), 0, N, K,
                                 _status(x2.device))

    @staticmethod
    def backward(ctx, dy):
        from rl_project_b200.ops._ext import native

        lin = ctx.lin
        N, K = lin.weight_shape
        dx = native().nf4_gemm(dy.contiguous(), lin.weight_packed, lin.weight_absmax.float(), lin._table(dy.device), 1, N, K,
                               _status(dy.device))
        return dx, None


class NF4Linear(nn.Module):
    def __init__(self, original: nn.Linear):
        super().__init__()
        packed, absmax, shape = quantize_nf4(original.weight.data)
        dev = original.weight.device
        self.register_buffer("weight_packed", packed.to(dev))
        self.register_buffer("weight_absmax", absmax.to(dev))
        self.weight_shape = tuple(shape)
        self.in_features = original.in_features
        self.out_features = original.out_features
        self.bias = (nn.Parameter(original.bias.detach().clone(), requires_grad=False)
                     if original.bias is not None else None)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return dequantize_nf4(self.weight_packed, self.weight_absmax, torch.Size(self.weight_shape), dtype)

    def _table(self, device: torch.device) -> torch.Tensor:
        t = getattr(self, "_table_dev", None)
        if t is None or t.device != device:
            t = self._table_dev = NF4_TABLE.to(device)
        return t

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if (_NF4_GEMM and x.is_cuda and x.dtype == torch.bfloat16 and self.in_features % 64 == 0
                and self.out_features % 8 == 0):
            shape = x.shape
            y = _NF4Matmul.apply(x.reshape(-1, shape[-1]).contiguous(), self).view(*shape[:-1], self.out_features)
            return y + self.bias.to(y.dtype) if self.bias is not None else y
        w = self.dequantized_weight(x.dtype if x.is_cuda else torch.float32).to(x.device, x.dtype)
        b = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, w, b)

    def memory_bytes(self) -> int:
        return self.weight_packed.numel() + self.weight_absmax.numel() * 4


def quantization_report(model: nn.Module) -> dict:
    layers = packed = fp16 = 0
    for m in model.modules():
        if isinstance(m, NF4Linear):
            layers += 1
            packed += m.memory_bytes()
            fp16 += m.in_features * m.out_features * 2
    return {"nf4_layers": layers, "nf4_bytes": packed, "fp16_equivalent_bytes": fp16,
            "compression_ratio": fp16 / packed if packed else 0.0}
