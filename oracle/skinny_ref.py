"""Oracle for the skinny weight-only linear y[M, N] = x[M, K] . W[N, K]^T (numpy, CPU).

Restates (reference paths inside the byteprof project):
  quantize_rowwise_int8   byteprof/quant/triton_int8.py:50-55
  dequantize              byteprof/optim/skinny.py:209-217 (bf16, int8 and int4 kinds)
  quantize_int4, pack_int4, unpack_int4
                          byteprof/optim/skinny.py:172-206 (int4 in groups of 128, tile-major packing)
  linear_ref              the fp32 dequantize-then-matmul reference of tests/test_skinny.py:38 and
                          tests/test_quant_int8.py:197-199
  nerr                    tests/test_skinny.py:34-40 (componentwise error, tolerance 4e-3)
  close_int8              tests/test_quant_int8.py:202-205
All arrays are float32 numpy arrays holding the values (bf16 tensors are passed as their exact
float32 values).
"""

from __future__ import annotations

import numpy as np

from .bf16 import round_bf16

TOL_COMPONENTWISE = 4e-3  # tests/test_skinny.py:17


def quantize_rowwise_int8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-row int8 of bf16-valued w [N, K] -> (q int8 [N, K], scale [N] bf16-valued float32).

    The scale max|row| / 127 (fp32 division, clamped below at 1e-12) is rounded to bf16 first, and q is
    rounded (half to even) against that stored scale, then clamped to [-127, 127]."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1).astype(np.float32)
    scale = round_bf16(np.maximum(amax / np.float32(127.0), np.float32(1e-12)))
    q = np.rint(w / scale[:, None]).clip(-127, 127).astype(np.int8)
    return q, scale


GROUP = 128


def quantize_int4(w: np.ndarray, tile_rows: int = 32) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Asymmetric int4 of bf16-valued w [N, K] in groups of 128 along K -> (packed uint8 [T, G, R, 64],
    scale [G, N] bf16-valued float32, zero [G, N] float16). Per group, in fp32: scale = max(
    (max - min) / 15, 1e-6) rounded to bf16; zero = -min / scale rounded to fp16; q = round-half-even(
    w / scale + zero) clamped to 0..15."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    if k % GROUP:
        raise ValueError("int4 needs K % 128 == 0")
    wg = w.reshape(n, k // GROUP, GROUP)
    lo, hi = wg.min(axis=-1), wg.max(axis=-1)
    scale = round_bf16(np.maximum((hi - lo) / np.float32(15.0), np.float32(1e-6)))
    zero = (-lo / scale).astype(np.float16)
    q = np.clip(np.rint(wg / scale[..., None] + zero.astype(np.float32)[..., None]), 0, 15).astype(np.uint8)
    return pack_int4(q.reshape(n, k), tile_rows), np.ascontiguousarray(scale.T), np.ascontiguousarray(zero.T)


def pack_int4(q: np.ndarray, tile_rows: int = 32) -> np.ndarray:
    """Codes [N, K] (0..15) -> [T, G, R, 64]: in each group of 128 along K, byte j = code j | code (j+64) << 4;
    rows padded with zeros to a multiple of R; tile t, group g is the R x 64 block [t, g]."""
    n, k = q.shape
    t = -(-n // tile_rows)
    qp = np.zeros((t * tile_rows, k), np.uint8)
    qp[:n] = q
    grp = qp.reshape(t, tile_rows, k // GROUP, GROUP)            # [T, R, G, 128]
    b = grp[..., :64] | (grp[..., 64:] << 4)                     # [T, R, G, 64]
    return np.ascontiguousarray(b.transpose(0, 2, 1, 3))         # [T, G, R, 64]


def unpack_int4(packed: np.ndarray, n: int) -> np.ndarray:
    """[T, G, R, 64] -> codes [N, K]."""
    t, ng, r, _ = packed.shape
    b = packed.transpose(0, 2, 1, 3)                             # [T, R, G, 64]
    codes = np.concatenate([b & 0xF, b >> 4], axis=-1)           # [T, R, G, 128]
    return codes.reshape(t * r, ng * GROUP)[:n]


def dequantize(kind: str, w: np.ndarray, scale: np.ndarray | None = None,
               zero: np.ndarray | None = None) -> np.ndarray:
    """fp32 reference weights [N, K]: bf16 -> the values; int8 -> q * scale (exact in fp32);
    int4 -> (q - zero) * scale per group, in fp32."""
    if kind == "bf16":
        return np.asarray(w, dtype=np.float32)
    if kind == "int8":
        return np.asarray(w, dtype=np.float32) * np.asarray(scale, dtype=np.float32)[:, None]
    if kind == "int4":
        ng, n = scale.shape
        codes = unpack_int4(w, n).astype(np.float32).reshape(n, ng, GROUP)
        d = (codes - np.asarray(zero, np.float32).T[..., None]) * np.asarray(scale, np.float32).T[..., None]
        return d.reshape(n, ng * GROUP)
    raise ValueError(f"unknown weight kind {kind!r}")


def linear_ref(x: np.ndarray, w_deq: np.ndarray, exact: bool = False) -> np.ndarray:
    """x [M, K] . w_deq [N, K]^T. exact=True accumulates in float64, else float32 (BLAS)."""
    if exact:
        return np.asarray(x, np.float64) @ np.asarray(w_deq, np.float64).T
    return (np.asarray(x, np.float32) @ np.asarray(w_deq, np.float32).T).astype(np.float64)


def nerr(y: np.ndarray, x: np.ndarray, w_deq: np.ndarray) -> float:
    """max_ij |y - ref|_ij / (|x| |W|^T)_ij: error relative to the sum of the absolute terms."""
    ref = linear_ref(x, w_deq)
    scale = np.maximum(linear_ref(np.abs(x), np.abs(w_deq)), 1e-30)
    return float((np.abs(np.asarray(y, np.float64) - ref) / scale).max())


def close_int8(y: np.ndarray, ref: np.ndarray) -> bool:
    """max|y - ref| <= 0.01 * max|ref| + 1e-3 (bf16 output rounding plus accumulation order)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return bool(np.abs(y - ref).max() <= 0.01 * np.abs(ref).max() + 1e-3)


def rel_normwise(a: np.ndarray, b: np.ndarray) -> float:
    """max|a - b| / max|b| (tests/test_fused_kernels_gpu.py:37-39)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rms_bound_ratio(y: np.ndarray, ref: np.ndarray) -> float:
    """max|y - ref| / rms(ref): the bf16 parity bar is <= 1e-2."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.abs(y - ref).max() / max(rms, 1e-30))
