"""int8 weight-only GEMV (one activation row) and the per-row int8 quantizer.

Same API as byteprof/quant/triton_int8.py:33-55: `gemv_int8(x, w, scale, cfg=None, out=None)`
and `quantize_rowwise_int8(w)`. The GEMV runs the skinny kernel family with M = 1
(bp_gemv_int8); `cfg` is accepted and ignored.
"""

from __future__ import annotations

import torch

from .. import _lib

DEFAULT_CFG = (2, 1024, 2)  # the reference's Triton (BN, BK, warps); no meaning for the B200 kernel


def default_cfg(n_out: int) -> tuple[int, int, int]:
    return (2, 512, 2) if n_out <= 1024 else DEFAULT_CFG


def gemv_int8(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, cfg: tuple[int, int, int] | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """x: [1, K] bf16, w: [N, K] int8, scale: [N] bf16 -> [1, N] (dtype of `out`, default x.dtype)."""
    n, k = w.shape
    if x.numel() != k:
        raise ValueError(f"x must hold one row of K = {k} values, got shape {tuple(x.shape)}")
    if w.dtype != torch.int8 or scale.numel() != n:
        raise ValueError("w must be int8 [N, K] and scale [N]")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"x must be bf16, got {x.dtype}")
    y = out if out is not None else torch.empty(1, n, dtype=x.dtype, device=x.device)
    if y.numel() != n or not y.is_contiguous():
        raise ValueError("out must be a contiguous [1, N] tensor")
    if n == 0:
        return y
    _lib.require_cuda(x, w, scale, y)
    x = x.contiguous()
    if scale.dtype != torch.bfloat16:
        scale = scale.to(torch.bfloat16)
    with _lib.on_device(x):
        ws, ws_bytes = _lib.skinny_workspace(x.device, 1, n, k, _lib.BP_DTYPE_INT8)
        _lib.call("bp_gemv_int8", x.data_ptr(), w.contiguous().data_ptr(), scale.contiguous().data_ptr(), y.data_ptr(),
                  _lib.dtype_code(y.dtype), n, k, ws, ws_bytes, _lib.stream_of(x))
    return y


def quantize_rowwise_int8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-row int8: w ~ q * scale[:, None]; scale in the weight's dtype.

    The scale max|row| / 127 (clamped below at 1e-12) is rounded to the weight dtype before q is
    computed, so q is quantized against the scale that is stored (byteprof/quant/triton_int8.py:50-55).
    Offline weight preparation: runs wherever w lives."""
    wf = w.float()
    scale = (wf.abs().amax(dim=1) / 127.0).clamp_min(1e-12).to(w.dtype)
    q = torch.round(wf / scale.float()[:, None]).clamp_(-127, 127).to(torch.int8)
    return q.contiguous(), scale
