"""Seeded inputs and torch <-> oracle conversions shared by the tests."""

from __future__ import annotations

import numpy as np
import torch


def to_np(t: torch.Tensor) -> np.ndarray:
    """Exact float32 numpy copy of a bf16 / fp32 / int tensor (on any device)."""
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.numpy().copy()


def make_weights(kind: str, n: int, k: int, seed: int = 0, device: str = "cuda", std: float = 0.02):
    """W ~ N(0, std) in bf16 from a seeded generator (the reference tests' `make`,
    tests/test_skinny.py:23-31); int8 adds the per-row quantization, int4 the group-128 quantization
    in the tile-major format. Returns (w_bf16, args)."""
    from byteprof_b200.quant.int8 import quantize_rowwise_int8

    from byteprof_b200.optim.skinny import quantize_int4

    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn(n, k, generator=g, device=device) * std).to(torch.bfloat16)
    if kind == "bf16":
        return w, (w,)
    if kind == "int4":
        return w, quantize_int4(w)
    q, s = quantize_rowwise_int8(w)
    return w, (q, s)


def deq_np(kind: str, args) -> np.ndarray:
    from oracle import skinny_ref

    if kind == "bf16":
        return skinny_ref.dequantize("bf16", to_np(args[0]))
    if kind == "int4":
        return skinny_ref.dequantize("int4", args[0].cpu().numpy(), to_np(args[1]), args[2].cpu().numpy())
    return skinny_ref.dequantize("int8", to_np(args[0]), to_np(args[1]))


def randn(*shape, seed: int, device: str = "cuda", dtype=torch.bfloat16, scale: float = 1.0) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=device) * scale).to(dtype)


def bf16_step_close(a, b, min_exact: float = 0.99) -> tuple[bool, float, float]:
    """bf16 outputs a vs float reference b: every element within one bf16 step of b
    (|a - b| <= 2^-7 |b| + 1e-6 max|b|), and at least `min_exact` of them equal to b rounded to bf16.
    Returns (ok, worst step fraction, exact fraction)."""
    from oracle.bf16 import round_bf16

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    tol = np.abs(b) * 2.0**-7 + 1e-6 * max(np.abs(b).max(), 1e-30)
    worst = float((np.abs(a - b) / tol).max())
    exact = float(np.mean(a == round_bf16(b.astype(np.float32))))
    return worst <= 1.0 and exact >= min_exact, worst, exact
