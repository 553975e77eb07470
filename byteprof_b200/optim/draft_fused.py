"""Fused mLSTM verification kernels: `multistep_fw`, `lazy_commit`, `accept`.

Same API as byteprof/optim/draft_fused.py:27-62, on one sm_100a kernel (bp_mlstm_scan) that keeps the
recurrent state on chip across all positions:
  * multistep_fw(cur, q, k, v, i, f, h, nstart, mstart, eps): h for T positions from the state `cur`
    (not modified); the start n and m are copied to nstart / mstart.
  * lazy_commit(cur, k, v, i, f, length, nstart, mstart): cur <- the state after positions 0..L,
    L read on the device from `length` (so the count can change between CUDA-graph replays),
    recomputed from the start state (c from cur, n and m from nstart / mstart).
  * accept(ids, tok, out, s, smax): draft acceptance on the device.
State layouts as the reference: c (1, NH, DQ, DV), n (1, NH, DQ), m (1, NH, 1), fp32, contiguous;
q, k (T, NH, DQ), v (T, NH, DV), i, f (T, NH, 1), h (>= T, NH, DV); only the position stride may
differ from the contiguous one (q and k must share it). qk_scale = DQ ** -0.5.
Supported head dims: DQ in {64, 128, 256, 512}, DV a multiple of 16 (the reference's wrapper
accepted DQ of one or two library blocks, draft_fused.py:19-22); others raise NotImplementedError.
"""

from __future__ import annotations

import torch

from .. import _lib

BV = 16
SUPPORTED_DQ = (64, 128, 256, 512)


def _geometry(q: torch.Tensor, v: torch.Tensor) -> tuple[int, int, int]:
    _, nh, dq = q.shape
    dv = v.shape[-1]
    if dq not in SUPPORTED_DQ or dv % BV:
        raise NotImplementedError(f"the fused kernel needs head_dim_qk in {SUPPORTED_DQ} and head_dim_v a multiple "
                                  f"of {BV} (got {dq}, {dv})")
    return nh, dq, dv


def _check_state(cur, nh: int, dq: int, dv: int) -> None:
    c, n, m = cur
    if tuple(c.shape) != (1, nh, dq, dv) or tuple(n.shape) != (1, nh, dq) or m.numel() != nh:
        raise ValueError("state must be c (1, NH, DQ, DV), n (1, NH, DQ), m (1, NH, 1)")
    for t in cur:
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("the state tensors must be contiguous fp32")


def _check_seq(q, k, v, i, f, h, nh: int, dq: int, dv: int) -> None:
    if k.shape[1:] != (nh, dq) or v.shape[1:] != (nh, dv) or i.shape[1] != nh or f.shape[1] != nh:
        raise ValueError("q, k (T, NH, DQ), v (T, NH, DV), i, f (T, NH, 1) expected")
    if q is not None and (q.stride(1) != dq or q.stride(2) != 1 or q.stride(0) != k.stride(0)):
        raise ValueError("q and k need contiguous (NH, DQ) rows and the same position stride")
    if k.stride(1) != dq or k.stride(2) != 1 or v.stride(1) != dv or v.stride(2) != 1:
        raise ValueError("k, v need contiguous head rows")
    if i.stride(1) != 1 or f.stride(1) != 1 or i.stride(0) != f.stride(0) or i.dtype != f.dtype:
        raise ValueError("i and f need unit head stride, the same position stride and dtype")
    if h is not None and (h.shape[1:] != (nh, dv) or h.stride(1) != dv or h.stride(2) != 1):
        raise ValueError("h must be (>= T, NH, DV) with contiguous head rows")


def multistep_fw(cur: tuple[torch.Tensor, ...], q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, i: torch.Tensor,
                 f: torch.Tensor, h: torch.Tensor, nstart: torch.Tensor, mstart: torch.Tensor, eps: float) -> None:
    """T = q.shape[0] positions from `cur` (not modified); h receives the outputs; nstart (NH, DQ) and
    mstart (NH,) receive the start n and m."""
    nh, dq, dv = _geometry(q, v)
    _check_state(cur, nh, dq, dv)
    _check_seq(q, k, v, i, f, h, nh, dq, dv)
    t = q.shape[0]
    if h.shape[0] < t:
        raise ValueError("h has fewer positions than q")
    _lib.require_cuda(*cur, q, k, v, i, f, h, nstart, mstart)
    with _lib.on_device(q):
        _lib.call("bp_mlstm_scan", cur[0].data_ptr(), cur[1].data_ptr(), cur[2].data_ptr(), q.data_ptr(), k.data_ptr(),
                  v.data_ptr(), i.data_ptr(), f.data_ptr(), h.data_ptr(), None, None, None, nstart.data_ptr(),
                  mstart.data_ptr(), None, t, nh, dq, dv, q.stride(0), v.stride(0), i.stride(0), h.stride(0),
                  _lib.dtype_code(q.dtype), _lib.dtype_code(i.dtype), dq ** -0.5, eps, _lib.stream_of(q))


def lazy_commit(cur: tuple[torch.Tensor, ...], k: torch.Tensor, v: torch.Tensor, i: torch.Tensor, f: torch.Tensor,
                length: torch.Tensor, nstart: torch.Tensor, mstart: torch.Tensor) -> None:
    """cur <- the state after positions 0..L (L = `length`, a 0-d device int64), from the start state."""
    nh, dq, dv = _geometry(k, v)
    _check_state(cur, nh, dq, dv)
    _check_seq(None, k, v, i, f, None, nh, dq, dv)
    if length.dtype != torch.int64 or length.numel() != 1:
        raise ValueError("length must be a one-element int64 device tensor")
    _lib.require_cuda(*cur, k, v, i, f, length, nstart, mstart)
    with _lib.on_device(k):
        # q is not read for the state: k stands in so that every prefetched address is valid.
        _lib.call("bp_mlstm_scan", cur[0].data_ptr(), nstart.data_ptr(), mstart.data_ptr(), k.data_ptr(),
                  k.data_ptr(), v.data_ptr(), i.data_ptr(), f.data_ptr(), None, cur[0].data_ptr(), cur[1].data_ptr(),
                  cur[2].data_ptr(), None, None, length.data_ptr(), k.shape[0], nh, dq, dv, k.stride(0), v.stride(0),
                  i.stride(0), 0, _lib.dtype_code(k.dtype), _lib.dtype_code(i.dtype), dq ** -0.5, 0.0,
                  _lib.stream_of(k))


def accept(ids: torch.Tensor, tok: torch.Tensor, out: torch.Tensor, s: int, smax: int) -> None:
    """out[:s] <- tok[:s], out[smax] <- accepted length (int64 tensors)."""
    for t in (ids, tok, out):
        if t.dtype != torch.int64 or not t.is_contiguous():
            raise ValueError("ids, tok and out must be contiguous int64")
    if ids.numel() < s or tok.numel() < s or out.numel() <= smax:
        raise ValueError("ids/tok need s entries and out smax + 1")
    _lib.require_cuda(ids, tok, out)
    with _lib.on_device(out):
        _lib.call("bp_mlstm_accept", ids.data_ptr(), tok.data_ptr(), out.data_ptr(), s, smax, _lib.stream_of(out))
