"""The reference's CPU implementation of the hot path, timed as the CPU baseline (torch on the host).

  linear_cpu   byteprof/optim/skinny_linear.py:67-68 and byteprof/quant/integrate.py:45: on a
               non-CUDA tensor the reference runs F.linear on the weights dequantized to the
               activation dtype (bf16 here).
  mlstm_step_cpu  the eager torch mLSTM step in the library formulation (the oracle's step,
               oracle/mlstm_ref.py), on torch CPU tensors in fp32 with the bf16 casts.
Only bench.py's cpu_baseline / --impl reference legs use this module.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def linear_cpu(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor | None = None) -> torch.Tensor:
    """y = x . W^T with W bf16 [N, K], or int8 [N, K] dequantized with scale [N] to x's dtype."""
    if scale is not None:
        w = w.to(x.dtype) * scale.to(x.dtype)[:, None]
    return F.linear(x, w)


def _r(t: torch.Tensor, bf16: bool) -> torch.Tensor:
    return t.to(torch.bfloat16).float() if bf16 else t


def mlstm_step_cpu(c, n, m, q, k, v, i, f, qk_scale: float, eps: float, bf16: bool = True):
    """One position for all heads on torch CPU tensors (c [NH, DQ, DV], n [NH, DQ], m [NH], q, k
    [NH, DQ], v [NH, DV], i, f [NH], fp32 holding the input values). Returns (h, c, n, m)."""
    f_log = torch.log(torch.sigmoid(f))
    m_new = torch.maximum(f_log + m, i)
    max_val = _r(torch.exp(-m_new), bf16)
    f_act = _r(torch.exp(f_log + m - m_new), bf16)
    i_act = _r(torch.exp(i - m_new), bf16)
    kv = _r(k[:, :, None] * v[:, None, :], bf16)
    c = f_act[:, None, None] * c + _r(i_act[:, None, None] * kv, bf16)
    n = f_act[:, None] * n + _r(i_act[:, None] * k, bf16)
    qs = _r(q * _r(torch.tensor(qk_scale), bf16), bf16)
    hn = _r(qs[:, :, None] * _r(c, bf16), bf16).sum(1)
    qn = _r(qs * _r(n, bf16), bf16).sum(1)
    h = _r(hn / (torch.maximum(qn.abs(), max_val) + eps)[:, None], bf16)
    return h, c, n, m_new
