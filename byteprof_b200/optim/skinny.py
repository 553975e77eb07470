"""Skinny weight-only matmul y[M, N] = x[M, K] . W[N, K]^T on the sm_100a kernels.

Same API and error behaviour as byteprof/optim/skinny.py:136-166 (`skinny_mm`) and 209-217
(`dequantize`). Weight formats:
  bf16  W: [N, K] bf16
  int8  W: [N, K] int8 with scale [N] (bf16): w ~ q * scale[n]   (byteprof_b200.quant.int8)
fp32 accumulation; the output has the dtype of `out` (bf16 by default, fp32 gives the unrounded
accumulator). The reference's int4 tile-major format (uint8 weights) is not built yet and raises
NotImplementedError.
"""

from __future__ import annotations

import torch

from .. import _lib

GROUP = 128
MAX_M = 64  # SkinnyLinear sends at most this many rows to the kernel (byteprof/optim/skinny.py:32)


def get_cfg(kind: str, n: int, k: int, bm: int) -> None:
    """The reference's Triton tile table (skinny.py:93-108) has no counterpart: the B200 kernels
    choose their tiling and split-K from the shape and the SM count. Kept so callers still import."""
    return None


def _kind(w: torch.Tensor) -> str:
    if w.dtype == torch.bfloat16:
        return "bf16"
    if w.dtype == torch.int8:
        return "int8"
    if w.dtype == torch.uint8:
        return "int4"
    raise ValueError(f"unsupported weight dtype {w.dtype}")


def skinny_mm(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor | None = None,
              zero: torch.Tensor | None = None, out: torch.Tensor | None = None,
              cfg: tuple[int, ...] | None = None) -> torch.Tensor:
    """x: [M, K] bf16 (contiguous); w: bf16 [N, K] | int8 [N, K] + scale [N]. `cfg` is accepted and ignored."""
    if x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [M, K] tensor")
    m, k = x.shape
    kind = _kind(w)
    if kind == "bf16":
        n = w.shape[0]
        if w.dim() != 2 or w.shape[1] != k:
            raise ValueError("K mismatch")
    elif kind == "int8":
        n = w.shape[0]
        if scale is None or w.dim() != 2 or w.shape[1] != k:
            raise ValueError("int8 needs scale [N] and K to match")
        if scale.numel() != n:
            raise ValueError("int8 scale must have N entries")
    else:
        raise NotImplementedError("the int4 tile-major weight format is not built in byteprof_b200 yet")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"x must be bf16, got {x.dtype}")
    y = out if out is not None else torch.empty(m, n, dtype=x.dtype, device=x.device)
    if y.shape != (m, n) or (m > 0 and n > 0 and y.stride(1) != 1):
        raise ValueError(f"out must be [M, N] = [{m}, {n}] with unit column stride")
    if y.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out must be bf16 or fp32, got {y.dtype}")
    if m == 0 or n == 0 or k == 0:
        if k == 0:
            y.zero_()
        return y
    _lib.require_cuda(x, w, y, scale)
    if not w.is_contiguous() or (scale is not None and not scale.is_contiguous()):
        raise ValueError("w and scale must be contiguous")
    if scale is not None and kind == "int8" and scale.dtype != torch.bfloat16:
        scale = scale.to(torch.bfloat16)
    wcode = _lib.dtype_code(w.dtype)
    with torch.cuda.device(x.device):
        ws, ws_bytes = _lib.skinny_workspace(x.device, m, n, k, wcode)
        _lib.call("bp_skinny_mm", x.data_ptr(), k, w.data_ptr(), wcode, _lib.ptr(scale if kind == "int8" else None),
                  y.data_ptr(), y.stride(0), _lib.dtype_code(y.dtype), m, n, k, ws, ws_bytes, _lib.stream_of(x))
    return y


def dequantize(kind: str, w: torch.Tensor, scale: torch.Tensor | None = None,
               zero: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 weights [N, K] (the reference dequantizer; used by the prefill / fp32-activation path)."""
    if kind == "bf16":
        return w.float()
    if kind == "int8":
        return w.float() * scale.float()[:, None]
    raise NotImplementedError("the int4 tile-major weight format is not built in byteprof_b200 yet")
