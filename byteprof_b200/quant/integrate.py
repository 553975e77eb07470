"""Quantize a model's selected linears in place: `Int8Linear` and `apply_quantization`.

Same API as byteprof/quant/integrate.py:22-122:
  * `Int8Linear(lin)`: per-row int8 weights; one-row CUDA inputs run the int8 GEMV kernel
    (bp_gemv_int8), other row counts use the weights dequantized to the activation dtype with
    F.linear on the GPU (the reference's prefill path). Bias added as a separate op.
  * `apply_quantization(model, target, scheme, group_size, local_scheme, global_scheme, kernel)`:
    the reference's selection rule (byteprof_b200.quant.select); kernel="skinny" swaps in
    `SkinnyLinear`, the default kernel swaps int8_wo linears for `Int8Linear`. The default int4_wo
    path of the reference calls torchao (tinygemm), which is not part of this build: it raises.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from .int8 import gemv_int8, quantize_rowwise_int8
from .select import group_of, olmo_should_quantize, should_quantize


class Int8Linear(nn.Module):
    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        q, scale = quantize_rowwise_int8(lin.weight.data)
        self.register_buffer("q", q)
        self.register_buffer("scale", scale)
        # Bolmo's remote code reads `weight.dtype` when it sets up its cache: an empty parameter keeps
        # that working without holding the bf16 weights.
        self.weight = nn.Parameter(torch.empty(0, dtype=lin.weight.dtype, device=lin.weight.device),
                                   requires_grad=False)
        self.bias = lin.bias

    def dequantized(self, dtype: torch.dtype) -> torch.Tensor:
        return self.q.to(dtype) * self.scale.to(dtype)[:, None]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.in_features)
        if x2.shape[0] == 0:
            return x.new_empty(*x.shape[:-1], self.out_features)
        if not x2.is_cuda:
            raise ValueError("Int8Linear runs on CUDA tensors only (there is no CPU path)")
        if x2.shape[0] == 1 and x2.dtype == torch.bfloat16:
            y = gemv_int8(x2, self.q, self.scale)
            if self.bias is not None:
                y = y + self.bias
        else:
            y = F.linear(x2, self.dequantized(x.dtype), self.bias)
        return y.reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, int8 rowwise (sm_100a GEMV)"


def _swap(model: nn.Module, name: str, make) -> None:
    parent_name, _, child = name.rpartition(".")
    parent = model.get_submodule(parent_name) if parent_name else model
    setattr(parent, child, make(getattr(parent, child)))


def apply_quantization(model: nn.Module, target: str, scheme: str, group_size: int = 128,
                       local_scheme: str | None = None, global_scheme: str | None = None,
                       kernel: str = "default") -> dict[str, Any]:
    """Quantize every linear selected by the target's rule; returns statistics (reference keys)."""
    bolmo = hasattr(model.model, "local_encoder")
    pick = should_quantize if bolmo else olmo_should_quantize
    names = [n for n, m in model.named_modules() if isinstance(m, nn.Linear) and pick(n, target)]
    before = torch.cuda.memory_allocated() if torch.cuda.is_available() else 0

    def scheme_of(n: str) -> str:
        g = group_of(n)
        over = local_scheme if g == "local" else global_scheme if g == "global" else None
        return over or scheme

    by_scheme: dict[str, list[str]] = {}
    for n in names:
        by_scheme.setdefault(scheme_of(n), []).append(n)
    for sch, group_names in by_scheme.items():
        if kernel == "skinny":
            from ..optim.skinny_linear import SkinnyLinear

            for n in group_names:
                _swap(model, n, lambda lin, sch=sch: SkinnyLinear(lin, sch))
        elif sch == "int4_wo":
            raise NotImplementedError("the default int4_wo path (torchao tinygemm) is not part of byteprof_b200")
        elif sch == "int8_wo":
            for n in group_names:
                _swap(model, n, Int8Linear)
        else:
            raise ValueError(f"unknown scheme {sch!r}")
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    after = torch.cuda.memory_allocated() if torch.cuda.is_available() else 0
    stats: dict[str, Any] = {"target": target, "scheme": scheme, "local_scheme": local_scheme,
                             "global_scheme": global_scheme,
                             "group_size": group_size if "int4_wo" in by_scheme else None,
                             "n_linears": len(names), "gpu_mem_before_mib": before / 2**20,
                             "gpu_mem_after_mib": after / 2**20}
    if kernel != "default":
        stats["kernel"] = kernel
    return stats
