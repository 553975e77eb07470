"""Oracle for the fused mLSTM recurrence (numpy, CPU).

Restates byteprof/optim/mlstm_multistep.py:20-146 (the formulation of the library step
mlstm_kernels 2.0.6 `recurrent_step_fw_kernel`, which that file reproduces) for all heads at once:

  _gates                 mlstm_multistep.py:20-30
  one position           mlstm_multistep.py:64-86 (state update, h)
  multistep_fw           mlstm_multistep.py:33-85 (h only; the start n, m copied)
  lazy_commit            mlstm_multistep.py:89-133 (state after positions 0..L from the start state)
  accept                 mlstm_multistep.py:136-146

Precision model. fp32 inputs: everything in fp32. bf16 inputs (Triton 3.6 rules,
triton/language/semantic.py computation_type_impl; tl.sum keeps bf16, standard.py:270-293):
  * f_act, i_act, max_val are rounded to bf16 (`.to(DTYPE)`, mlstm_multistep.py:27-29);
  * k*v, i_act*(k*v) and i_act*k are bf16 x bf16 products, rounded to bf16; f_act*C and f_act*n are
    fp32 (bf16 x fp32 promotes to fp32), the sums fp32;
  * `f_act * C + x` and `f_act * n + x` are single fused multiply-adds: Triton compiles with
    enable_fp_fusion on by default, so a product feeding an add becomes one fma.rn.f32 (emulated here in
    float64, whose product of two float32 values is exact, then rounded once to float32);
  * q*qk_scale: the scalar is rounded to bf16, the product to bf16;
  * C and n are rounded to bf16 before the output dot products (`c0.to(DTYPE)`), and each product
    q*C, q*n is rounded to bf16. The reference then reduces these bf16 products in bf16 (layout
    dependent order); this oracle sums them exactly (float64) and rounds the sum to fp32, which is
    what the B200 kernel's fp32 accumulation approximates to fp32 rounding.
Transcendental gate values are evaluated in float64 and rounded to fp32 wherever the reference
holds an fp32 value (exp(-x), 1 + e, the reciprocal, log, f_log + m, m - ...), so the bf16 gate
values are the correctly rounded ones. The reference's approximate fp32 exp can round a gate value
one bf16 step differently with probability about 2^-13 per value.
"""

from __future__ import annotations

import numpy as np

from .bf16 import round_bf16

F32 = np.float32


def _r(a, bf16: bool):
    return round_bf16(a) if bf16 else np.asarray(a, dtype=F32)


def gates(f: np.ndarray, i: np.ndarray, m_old: np.ndarray, bf16: bool):
    """Per-head gate values for one position: (m_new, max_val, f_act, i_act), float32 arrays."""
    f = np.asarray(f, F32)
    i = np.asarray(i, F32)
    m_old = np.asarray(m_old, F32)
    e = np.exp(-f.astype(np.float64)).astype(F32)
    d = (F32(1.0) + e).astype(F32)
    sig = (F32(1.0) / d).astype(F32)
    f_log = np.log(sig.astype(np.float64)).astype(F32)
    s = (f_log + m_old).astype(F32)
    m_new = np.maximum(s, i).astype(F32)
    a = (s - m_new).astype(F32)
    max_val = _r(np.exp(-m_new.astype(np.float64)).astype(F32), bf16)
    f_act = _r(np.exp(a.astype(np.float64)).astype(F32), bf16)
    i_act = _r(np.exp((i - m_new).astype(F32).astype(np.float64)).astype(F32), bf16)
    return m_new, max_val, f_act, i_act


def fma32(a, b, c) -> np.ndarray:
    """float32 fused multiply-add a * b + c with one rounding (float64 product exact, sum rounded twice
    only when the float64 sum itself rounds, which for these magnitudes does not change the float32 result
    in practice)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(F32)


def step(state, q, k, v, i, f, qk_scale: float, eps: float, bf16: bool, want_h: bool = True):
    """One position for all heads.

    state = (C [NH, DQ, DV], n [NH, DQ], m [NH]) float32; q, k [NH, DQ], v [NH, DV], i, f [NH] as the
    float32 values of the inputs. Returns (h [NH, DV] float32 or None, new state)."""
    c, n, m = state
    m_new, max_val, f_act, i_act = gates(f, i, m, bf16)
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    kv = _r(k[:, :, None] * v[:, None, :], bf16)
    ikv = _r(i_act[:, None, None] * kv, bf16)
    c_new = fma32(f_act[:, None, None], c, ikv)
    n_new = fma32(f_act[:, None], n, _r(i_act[:, None] * k, bf16))
    h = None
    if want_h:
        qs = _r(q * _r(F32(qk_scale), bf16), bf16)
        hn = _r(qs[:, :, None] * _r(c_new, bf16), bf16).astype(np.float64).sum(axis=1).astype(F32)
        qn = _r(qs * _r(n_new, bf16), bf16).astype(np.float64).sum(axis=1).astype(F32)
        den = (np.maximum(np.abs(qn), max_val) + F32(eps)).astype(F32)
        h = _r((hn / den[:, None]).astype(F32), bf16)
    return h, (c_new, n_new, m_new)


def scan(state, q, k, v, i, f, qk_scale: float, eps: float, bf16: bool, n_steps: int | None = None,
         want_h: bool = True, keep_states: bool = False):
    """Positions 0..n_steps-1 from `state`.

    q, k [T, NH, DQ], v [T, NH, DV], i, f [T, NH]. Returns (h [n_steps, NH, DV] or None, final state,
    list of the states after every position if keep_states)."""
    T = q.shape[0] if n_steps is None else n_steps
    cur = tuple(np.asarray(s, F32).copy() for s in state)
    hs, states = [], []
    for t in range(T):
        h, cur = step(cur, q[t], k[t], v[t], i[t], f[t], qk_scale, eps, bf16, want_h)
        if want_h:
            hs.append(h)
        if keep_states:
            states.append(cur)
    h_all = np.stack(hs) if want_h and hs else None
    return h_all, cur, states


def multistep_fw(state, q, k, v, i, f, qk_scale: float, eps: float, bf16: bool):
    """h for every position (the state is not modified) and the start (n, m) copy."""
    h, _, _ = scan(state, q, k, v, i, f, qk_scale, eps, bf16)
    return h, np.asarray(state[1], F32).copy(), np.asarray(state[2], F32).copy()


def lazy_commit(start, k, v, i, f, length: int, bf16: bool):
    """The state after positions 0..length (clamped to the available positions)."""
    T = k.shape[0]
    n_steps = max(0, min(int(length) + 1, T))
    dummy_q = np.zeros_like(np.asarray(k, F32))
    _, cur, _ = scan(start, dummy_q, k, v, i, f, 1.0, 0.0, bf16, n_steps=n_steps, want_h=False)
    return cur


def accept(ids, tok, s: int, smax: int, out_len: int):
    """out[:s] <- tok[:s]; out[smax] <- number of leading drafts ids[1 + j] == tok[j], j < s - 1."""
    out = np.zeros(out_len, dtype=np.int64)
    n, alive = 0, True
    for j in range(s - 1):
        alive = alive and int(ids[1 + j]) == int(tok[j])
        n += int(alive)
    out[:s] = np.asarray(tok[:s], dtype=np.int64)
    out[smax] = n
    return out
