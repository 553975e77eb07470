"""`SkinnyLinear`: an nn.Linear drop-in that runs the sm_100a skinny kernels.

Same constructor, attributes and forward behaviour as byteprof/optim/skinny_linear.py:20-69:
  * schemes bf16_wo (keeps the bf16 weight Parameter) and int8_wo (per-row int8 `q` and bf16 `scale`
    buffers plus an empty `weight` Parameter that only carries the dtype, which Bolmo's cache setup
    reads) and int4_wo (the packed group-128 codes `q` with `scale` and `zero` buffers);
  * bf16 inputs of 1..MAX_M rows run the kernel, then the bias is added as a separate op;
  * empty inputs return an empty tensor;
  * larger inputs (prefill) and non-bf16 activations (the fp32 exactness runs) use the weights
    dequantized to the activation dtype with F.linear on the GPU, as the reference does.
Inputs must be CUDA tensors: there is no CPU path.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..quant.int8 import quantize_rowwise_int8
from . import skinny


class SkinnyLinear(nn.Module):
    def __init__(self, lin: nn.Linear, scheme: str):
        super().__init__()
        if scheme not in ("bf16_wo", "int8_wo", "int4_wo"):
            raise ValueError(f"unknown scheme {scheme!r}")
        self.scheme = scheme
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.bias = lin.bias
        w = lin.weight.data
        if scheme == "bf16_wo":
            self.weight = lin.weight
            self.scale = self.zero = None
            return
        self.weight = nn.Parameter(torch.empty(0, dtype=w.dtype, device=w.device), requires_grad=False)
        if scheme == "int8_wo":
            q, scale = quantize_rowwise_int8(w)
            self.register_buffer("q", q)
            self.register_buffer("scale", scale)
            self.zero = None
        else:
            packed, scale, zero = skinny.quantize_int4(w)
            self.register_buffer("q", packed)
            self.register_buffer("scale", scale)
            self.register_buffer("zero", zero)

    def _kind(self) -> str:
        return {"bf16_wo": "bf16", "int8_wo": "int8", "int4_wo": "int4"}[self.scheme]

    def dequantized(self, dtype: torch.dtype) -> torch.Tensor:
        if self.scheme == "bf16_wo":
            return self.weight
        return skinny.dequantize(self._kind(), self.q, self.scale, self.zero).to(dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.in_features)
        if x2.shape[0] == 0:
            return x.new_empty(*x.shape[:-1], self.out_features)
        if not x2.is_cuda:
            raise ValueError("SkinnyLinear runs on CUDA tensors only (there is no CPU path)")
        if x2.dtype == torch.bfloat16 and x2.shape[0] <= skinny.MAX_M:
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            w = self.weight if self.scheme == "bf16_wo" else self.q
            y = skinny.skinny_mm(x2, w, self.scale, self.zero)
            if self.bias is not None:
                y = y + self.bias
        else:
            y = F.linear(x2, self.dequantized(x.dtype), self.bias)
        return y.reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, {self.scheme}, skinny kernel (sm_100a)"
