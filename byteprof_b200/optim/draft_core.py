"""The mLSTM step of the minimal decode loop, and the fused T-position scan with the final state.

  * mlstm_step_into(prev, new, q, k, v, i, f, h, eps): one position from the state `prev` into the
    buffers `new` (byteprof/optim/draft_core.py:114-141, which wraps the library step kernel of
    mlstm_kernels 2.0.6). Batch 1: q, k (1, NH, DQ), v (1, NH, DV), i, f (1, NH, 1), h (1, NH, DV).
  * mlstm_scan(state_in, q, k, v, i, f, h, state_out, eps): T positions in one launch, h for every
    position and the state after the last one (multistep_fw + lazy_commit with L = T - 1 in a single
    pass; state_out may be state_in for the C tensor only when n and m go to other buffers).
Both run bp_mlstm_scan; layouts and head-dim limits as byteprof_b200.optim.draft_fused.
"""

from __future__ import annotations

import torch

from .. import _lib
from .draft_fused import _check_seq, _check_state, _geometry


def mlstm_scan(state_in: tuple[torch.Tensor, ...], q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               i: torch.Tensor, f: torch.Tensor, h: torch.Tensor | None, state_out: tuple[torch.Tensor, ...],
               eps: float) -> None:
    nh, dq, dv = _geometry(q, v)
    _check_state(state_in, nh, dq, dv)
    _check_state(state_out, nh, dq, dv)
    _check_seq(q, k, v, i, f, h, nh, dq, dv)
    if state_out[1].data_ptr() == state_in[1].data_ptr() or state_out[2].data_ptr() == state_in[2].data_ptr():
        raise ValueError("n and m of state_out must not alias state_in (other CTAs still read them)")
    t = q.shape[0]
    if h is not None and h.shape[0] < t:
        raise ValueError("h has fewer positions than q")
    _lib.require_cuda(*state_in, *state_out, q, k, v, i, f, h)
    with _lib.on_device(q):
        _lib.call("bp_mlstm_scan", state_in[0].data_ptr(), state_in[1].data_ptr(), state_in[2].data_ptr(),
                  q.data_ptr(), k.data_ptr(), v.data_ptr(), i.data_ptr(), f.data_ptr(), _lib.ptr(h),
                  state_out[0].data_ptr(), state_out[1].data_ptr(), state_out[2].data_ptr(), None, None, None,
                  t, nh, dq, dv, q.stride(0), v.stride(0), i.stride(0), 0 if h is None else h.stride(0),
                  _lib.dtype_code(q.dtype), _lib.dtype_code(i.dtype), dq ** -0.5, eps, _lib.stream_of(q))


def mlstm_step_into(prev: tuple[torch.Tensor, ...], new: tuple[torch.Tensor, ...], q: torch.Tensor, k: torch.Tensor,
                    v: torch.Tensor, i: torch.Tensor, f: torch.Tensor, h: torch.Tensor, eps: float) -> None:
    """One recurrence step from `prev` into `new` (batch 1), writing h."""
    if q.shape[0] != 1:
        raise NotImplementedError("mlstm_step_into supports batch 1 (the decode loop's shape)")
    mlstm_scan(prev, q, k, v, i, f, h, new, eps)
