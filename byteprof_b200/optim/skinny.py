"""Skinny weight-only matmul y[M, N] = x[M, K] . W[N, K]^T on the sm_100a kernels.

Same API and error behaviour as byteprof/optim/skinny.py:136-166 (`skinny_mm`), 172-206 (the int4
weight preparation) and 209-217 (`dequantize`). Weight formats:
  bf16  W: [N, K] bf16
  int8  W: [N, K] int8 with scale [N] (bf16): w ~ q * scale[n]   (byteprof_b200.quant.int8)
  int4  W: uint8 [ceil(N/R), K/128, R, 64] with scale [K/128, N] (bf16) and zero [K/128, N] (fp16):
        w ~ scale[g, n] * (q - zero[g, n]), q in 0..15, groups of 128 along K; inside a group, byte j of
        a row holds code j in its low nibble and code j + 64 in its high nibble, and the R rows of one
        group are one contiguous block (the reference's tile-major format, R = 32 by default).
fp32 accumulation; the output has the dtype of `out` (x's dtype by default; fp32 gives the unrounded
accumulator). Activations are bf16 (the reference's kernel input) or, beyond the reference, fp32 with bf16 or
int8 weights (the byte decoder's exactness mode; the CUDA-core kernel reads x as fp32).
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
    """x: [M, K] bf16 (or fp32 with bf16 / int8 weights), contiguous; w: bf16 [N, K] | int8 [N, K] + scale [N] |
    int4 tile-major uint8 + scale, zero [K/128, N]. `cfg` is accepted and ignored."""
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
        if (scale is None or zero is None or w.dim() != 4 or k % GROUP or w.shape[1] * GROUP != k
                or scale.shape[0] != w.shape[1]):
            raise ValueError("int4 needs packed [N/R, K/128, R, 64], scale/zero [K/128, N] and K % 128 == 0")
        n = scale.shape[1]
        if zero.shape != scale.shape:
            raise ValueError("int4 zero must have the shape of scale [K/128, N]")
    if x.dtype != torch.bfloat16 and not (x.dtype == torch.float32 and kind != "int4"):
        raise ValueError(f"x must be bf16 (or fp32 with bf16 / int8 weights), got {x.dtype}")
    y = out if out is not None else torch.empty(m, n, dtype=x.dtype, device=x.device)
    if y.shape != (m, n) or (m > 0 and n > 0 and y.stride(1) != 1):
        raise ValueError(f"out must be [M, N] = [{m}, {n}] with unit column stride")
    if y.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out must be bf16 or fp32, got {y.dtype}")
    if m == 0 or n == 0 or k == 0:
        if k == 0:
            y.zero_()
        return y
    _lib.require_cuda(x, w, y, scale, zero)
    if not w.is_contiguous() or (scale is not None and not scale.is_contiguous()):
        raise ValueError("w and scale must be contiguous")
    if kind == "int4":
        if scale.dtype != torch.bfloat16 or zero.dtype != torch.float16:
            raise ValueError("int4 scale must be bf16 and zero fp16 (as quantize_int4 makes them for bf16 weights)")
        with _lib.on_device(x):
            ws, ws_bytes = _lib.skinny_workspace(x.device, m, n, k, _lib.BP_DTYPE_INT4)
            _lib.call("bp_skinny_mm_int4", x.data_ptr(), k, w.data_ptr(), scale.data_ptr(), zero.contiguous().data_ptr(),
                      y.data_ptr(), y.stride(0), _lib.dtype_code(y.dtype), m, n, k, w.shape[2], ws, ws_bytes,
                      _lib.stream_of(x))
        return y
    if scale is not None and kind == "int8" and scale.dtype != torch.bfloat16:
        scale = scale.to(torch.bfloat16)
    wcode = _lib.dtype_code(w.dtype)
    if x.dtype == torch.float32:
        with _lib.on_device(x):
            _lib.call("bp_skinny_mm_xf32", x.data_ptr(), k, w.data_ptr(), wcode,
                      _lib.ptr(scale if kind == "int8" else None), y.data_ptr(), y.stride(0), _lib.dtype_code(y.dtype),
                      m, n, k, _lib.stream_of(x))
        return y
    with _lib.on_device(x):
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
    groups, n = scale.shape
    codes = unpack_int4(w, n).float().view(n, groups, GROUP) - zero.float().t().unsqueeze(-1)
    return (codes * scale.float().t().unsqueeze(-1)).view(n, groups * GROUP)


# ---- int4 weight preparation (offline; runs wherever w lives) -----------------------------------------


def quantize_int4(w: torch.Tensor, tile_rows: int = 32) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Asymmetric int4 in groups of 128 along K (byteprof/optim/skinny.py:172-184): per group,
    scale = (max - min) / 15 (at least 1e-6, rounded to w's dtype), zero = -min / scale (fp16), and
    q = round(w / scale + zero) clamped to 0..15. Returns (packed uint8 [ceil(N/R), K/128, R, 64],
    scale [K/128, N], zero [K/128, N])."""
    n, k = w.shape
    if k % GROUP:
        raise ValueError("int4 needs K % 128 == 0")
    groups = w.float().view(n, k // GROUP, GROUP)
    lo, hi = groups.amin(dim=-1), groups.amax(dim=-1)
    scale = ((hi - lo) / 15.0).clamp_min(1e-6).to(w.dtype)
    zero = (-lo / scale.float()).to(torch.float16)
    q = torch.round(groups / scale.float().unsqueeze(-1) + zero.float().unsqueeze(-1)).clamp_(0, 15).to(torch.uint8)
    return pack_int4(q.view(n, k), tile_rows), scale.t().contiguous(), zero.t().contiguous()


def pack_int4(q: torch.Tensor, tile_rows: int = 32) -> torch.Tensor:
    """Codes 0..15 [N, K] -> the tile-major [ceil(N/R), K/128, R, 64] (byteprof/optim/skinny.py:187-198):
    inside a group of 128, byte j = code j | code (j + 64) << 4; rows are padded with zeros to a
    multiple of R; the R rows of one group form one contiguous block."""
    n, k = q.shape
    tiles = -(-n // tile_rows)
    if tiles * tile_rows != n:
        q = torch.cat([q, q.new_zeros(tiles * tile_rows - n, k)])
    g = q.view(tiles * tile_rows, k // GROUP, GROUP)
    bytes_ = g[..., : GROUP // 2] | (g[..., GROUP // 2:] << 4)  # [rows, groups, 64]
    return bytes_.view(tiles, tile_rows, k // GROUP, GROUP // 2).transpose(1, 2).contiguous()


def unpack_int4(packed: torch.Tensor, n: int) -> torch.Tensor:
    """Inverse of pack_int4: [T, G, R, 64] -> codes [N, K] (byteprof/optim/skinny.py:201-206)."""
    tiles, groups, rows, _ = packed.shape
    p = packed.transpose(1, 2)  # [T, R, G, 64]
    codes = torch.cat([p & 0xF, p >> 4], dim=-1)  # [T, R, G, 128]
    return codes.reshape(tiles * rows, groups * GROUP)[:n]
