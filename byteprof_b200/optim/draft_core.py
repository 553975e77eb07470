"""Shared pieces of the drafting loop, with the names and signatures of byteprof/optim/draft_core.py.

A drafting round over S = K + 1 positions (the last emitted byte a0 and K drafted bytes): the encoder runs
all S positions and keeps the recurrent state after each one, the global model runs if a0 opened a patch,
the decoder predicts S tokens, L = the number of leading drafts the predictions confirm, the state after
position L becomes the current state, and the predictions p_1 .. p_{L+1} are emitted.

Device work:
  * mlstm_step_into(prev, new, q, k, v, i, f, h, eps): one recurrence position from `prev` into the buffers
    `new` (byteprof/optim/draft_core.py:114-141, which wraps the library step kernel of mlstm_kernels 2.0.6),
    on bp_mlstm_scan. Batch 1: q, k (1, NH, DQ), v (1, NH, DV), i, f (1, NH, 1), h (1, NH, DV).
  * mlstm_scan(state_in, q, k, v, i, f, h, state_out, eps): T positions in one launch, h for every position
    and the state after the last one (multistep_fw + lazy_commit with L = T - 1 in one pass).
  * commit_state(hist, cur, length): cur <- hist[length] with the length read on the device
    (draft_core.py:92-111), on bp_mlstm_commit_state for CUDA tensors. CPU tensors (the reference's toy
    models) are copied on the host as the reference does.
Host logic and torch references (draft_core.py:28-89, 144-248; pure torch, any device, parameterised by a
step function `step(prev, new, q1, k1, v1, i1, f1, h1)` such as mlstm_step_into with eps bound):
  accepted_length, accepted_length_t, scan_with_history, scan_without_history, lazy_commit_state,
  RoundEngine, Automaton, Stats, atom_of, choose_k, rounds_loop.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from typing import Any, Protocol

import torch

from .. import _lib
from .draft_fused import _check_seq, _check_state, _geometry

# ---------------------------------------------------------------------------------------------------
# acceptance
# ---------------------------------------------------------------------------------------------------


def accepted_length(ids: Sequence[int], toks: Sequence[int], k: int) -> int:
    """ids = [a0, d_1 .. d_K] (plain byte ids), toks = the predictions p_1 .. p_{K+1} (raw ids): the number of
    leading drafts d_j that equal p_j. A boundary-flagged prediction never equals a plain id, so it ends the
    accepted run."""
    for j in range(k):
        if ids[j + 1] != toks[j]:
            return j
    return k


def accepted_length_t(ids: torch.Tensor, tok: torch.Tensor, s: int) -> torch.Tensor:
    """`accepted_length` on tensors, without a host synchronisation: a 0-d integer tensor on ids' device.
    ids (>= S,), tok (>= S,); drafts ids[1:S] are compared with tok[:S-1]."""
    hit = (ids[1:s] == tok[:s - 1]).to(torch.int32)
    # the run of leading matches: a running product stays 1 until the first mismatch
    return torch.cumprod(hit, 0).sum()


# ---------------------------------------------------------------------------------------------------
# the recurrence over S positions
# ---------------------------------------------------------------------------------------------------


def scan_with_history(step: Callable, cur: tuple[torch.Tensor, ...], hist: tuple[torch.Tensor, ...], s: int,
                      q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, i: torch.Tensor, f: torch.Tensor,
                      hbuf: torch.Tensor) -> None:
    """S recurrence positions from `cur` (left unchanged) on precomputed projections; the state after position
    j goes into history slot j and the cell output into hbuf[j].

    cur   (c, n, m) of shapes (1, NH, DQ, DV), (1, NH, DQ), (1, NH, 1)
    hist  (C, N, M) slot tensors (Smax, 1, NH, DQ, DV), (Smax, 1, NH, DQ), (Smax, 1, NH, 1)
    q, k  (S, NH, DQ); v (S, NH, DV); i, f (S, NH, 1); hbuf (>= S, NH, DV)
    """
    prev = cur
    for j in range(s):
        slot = tuple(t[j] for t in hist)
        step(prev, slot, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], hbuf[j:j + 1])
        prev = slot


def scan_without_history(step: Callable, cur: tuple[torch.Tensor, ...], s: int, q: torch.Tensor, k: torch.Tensor,
                         v: torch.Tensor, i: torch.Tensor, f: torch.Tensor,
                         hbuf: torch.Tensor) -> tuple[torch.Tensor, ...]:
    """The lazy-commit form of `scan_with_history` (the torch reference of the fused multistep kernel): the same
    S positions writing only the cell outputs, through two ping-pong state buffers, `cur` unchanged. Returns a
    copy of the start state for `lazy_commit_state`."""
    start = tuple(t.clone() for t in cur)
    bufs = (tuple(torch.empty_like(t) for t in cur), tuple(torch.empty_like(t) for t in cur))
    prev = start
    for j in range(s):
        nxt = bufs[j & 1]
        step(prev, nxt, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], hbuf[j:j + 1])
        prev = nxt
    return start


def lazy_commit_state(step: Callable, cur: tuple[torch.Tensor, ...], start: tuple[torch.Tensor, ...],
                      length: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, i: torch.Tensor,
                      f: torch.Tensor) -> None:
    """cur <- the state after positions 0 .. L (L = `length`, a 0-d tensor), recomputed from `start` with the
    round's projections (the torch reference of the lazy-commit kernel; reads L on the host)."""
    bufs = (tuple(torch.empty_like(t) for t in cur), tuple(torch.empty_like(t) for t in cur))
    h = torch.empty(1, q.shape[1], v.shape[-1], dtype=q.dtype, device=q.device)
    prev = start
    for j in range(int(length) + 1):
        nxt = bufs[j & 1]
        step(prev, nxt, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], h)
        prev = nxt
    for dst, src in zip(cur, prev):
        dst.copy_(src)


def commit_state(hist: tuple[torch.Tensor, ...], cur: tuple[torch.Tensor, ...], length: torch.Tensor) -> None:
    """cur <- hist[length] for one layer's state (c, n, m); `length` is a one-element integer tensor on the
    state's device. On CUDA one launch of bp_mlstm_commit_state reads the slot on the device (no host
    synchronisation; capturable in a CUDA graph, the slot may change between replays); a slot outside the
    history fills cur with NaN. CPU tensors are copied on the host, as the reference does for its CPU toy
    models."""
    if len(hist) != 3 or len(cur) != 3:
        raise ValueError("hist and cur must each hold (c, n, m)")
    if not cur[0].is_cuda:
        slot = int(length)
        for h, c in zip(hist, cur):
            c.copy_(h[slot])
        return
    slots = hist[0].shape[0]
    for h, c in zip(hist, cur):
        if h.dtype != torch.float32 or c.dtype != torch.float32 or not h.is_contiguous() or not c.is_contiguous():
            raise ValueError("commit_state takes contiguous fp32 history and state tensors")
        if h.shape[0] != slots or h[0].numel() != c.numel():
            raise ValueError("each history tensor must hold `slots` copies of its state tensor")
    if length.dtype not in (torch.int32, torch.int64) or length.numel() != 1:
        raise ValueError("length must be a one-element int32 or int64 tensor")
    _lib.require_cuda(*hist, *cur, length)
    with _lib.on_device(cur[0]):
        _lib.call("bp_mlstm_commit_state", hist[0].data_ptr(), hist[1].data_ptr(), hist[2].data_ptr(),
                  cur[0].data_ptr(), cur[1].data_ptr(), cur[2].data_ptr(), cur[0].numel(), cur[1].numel(),
                  cur[2].numel(), length.data_ptr(), length.element_size(), slots, _lib.stream_of(cur[0]))


# ---------------------------------------------------------------------------------------------------
# the mLSTM step and scan on the sm_100a kernel
# ---------------------------------------------------------------------------------------------------


def mlstm_scan(state_in: tuple[torch.Tensor, ...], q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               i: torch.Tensor, f: torch.Tensor, h: torch.Tensor | None, state_out: tuple[torch.Tensor, ...],
               eps: float) -> None:
    """T = q.shape[0] positions from state_in; h (>= T, NH, DV) receives every position's output and state_out
    the state after the last one. state_out may share the C tensor with state_in; n and m must not alias.
    Layouts and head-dim limits as byteprof_b200.optim.draft_fused."""
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
    """One recurrence position from `prev` into `new` (batch 1), writing h; `prev` is not modified (its C may
    be `new`'s C only when n and m go to other buffers)."""
    if q.shape[0] != 1:
        raise NotImplementedError("mlstm_step_into supports batch 1 (the decode loop's shape)")
    mlstm_scan(prev, q, k, v, i, f, h, new, eps)


# ---------------------------------------------------------------------------------------------------
# the host round loop
# ---------------------------------------------------------------------------------------------------


class RoundEngine(Protocol):
    k_values: tuple[int, ...]  # the draft lengths K the engine has a graph for, 0 included

    def run_round(self, k: int, boundary: bool, ids: Sequence[int], subs: Sequence[int]) -> tuple[Sequence[int], int]:
        """Encoder, global model (when `boundary`) and decoder over the K + 1 inputs: returns the K + 1
        predicted raw ids and L as the device computed it."""


class Automaton(Protocol):
    def step(self, state: int, byte: int) -> tuple[int, int]: ...


class Stats:
    """Round tallies of a drafting run."""

    def __init__(self) -> None:
        self.rounds = 0
        self.emitted = 0
        self.by_k: dict[int, int] = {}
        self.l_hist: dict[int, int] = {}
        self.global_calls = 0
        self.draft_us = 0.0

    def dump(self) -> dict:
        return {"rounds": self.rounds, "emitted": self.emitted, "by_k": dict(self.by_k), "l_hist": dict(self.l_hist),
                "global_calls": self.global_calls, "bytes_per_round": self.emitted / max(self.rounds, 1)}


def atom_of(raw: int, byte_offset: int, boundary_offset: int) -> int | None:
    """A raw token id -> the atom (byte | boundary flag << 8), or None for ids that are not bytes."""
    flagged = raw >= boundary_offset
    b = (raw - boundary_offset if flagged else raw) - byte_offset
    if not 0 <= b < 256:
        return None
    return b | (256 if flagged else 0)


def choose_k(draft_len: int, k_values: Sequence[int], k_cap: int) -> int:
    """The largest available K that is at most the draft's length and the cap (0 when none is)."""
    fits = [kv for kv in k_values if 0 < kv <= min(draft_len, k_cap)]
    return max(fits, default=0)


def rounds_loop(engine: RoundEngine, automaton: Automaton, drafter: Any, *, state: int, sub: int, raw: int,
                tokens: list[int], n_tok: int, stop_len: int, eos_ids: tuple[int, ...], bpe_end: int,
                byte_offset: int, boundary_offset: int, k_max: int, stats: Stats | None = None,
                on_round: Callable[[dict], None] | None = None, k_cap_for: Callable[[Any], int] | None = None) -> int:
    """Drafting rounds until `stop_len` tokens or an EOS id. `raw` is the last emitted raw id a0, `state` / `sub`
    the automaton state and subword id after it. Each emitted id goes, without its boundary flag, into
    tokens[n_tok:]. Returns the new n_tok. The device's accepted length must equal the host's."""
    ks = engine.k_values
    while True:
        if raw == bpe_end:
            raise RuntimeError("model produced <bpe_token_end>; unsupported at batch 1")
        boundary = raw >= boundary_offset
        want = drafter is not None and k_max > 0 and len(ks) > 1
        draft = drafter.propose(k_max) if want else []
        cap = k_max if k_cap_for is None else k_cap_for(drafter)
        k = choose_k(len(draft), ks, cap)
        ids = [raw - boundary_offset if boundary else raw]
        subs, states = [sub], [state]
        st = state
        for atom in draft[:k]:
            byte_id = (atom & 255) + byte_offset
            st, sb = automaton.step(st, byte_id)
            ids.append(byte_id)
            subs.append(sb)
            states.append(st)
        preds, l_dev = engine.run_round(k, boundary, ids, subs)
        n_acc = accepted_length(ids, preds, k)
        if n_acc != l_dev:
            raise RuntimeError(f"host and device disagree on the accepted length ({n_acc} vs {l_dev})")
        if stats is not None:
            stats.rounds += 1
            stats.by_k[k] = stats.by_k.get(k, 0) + 1
            stats.l_hist[n_acc] = stats.l_hist.get(n_acc, 0) + 1
            stats.global_calls += int(boundary)
        emitted: list[int] = []
        done = False
        for r in (int(p) for p in preds[:n_acc + 1]):
            if r == bpe_end:
                raise RuntimeError("model produced <bpe_token_end>; unsupported at batch 1")
            tokens[n_tok] = r - boundary_offset if r >= boundary_offset else r
            n_tok += 1
            emitted.append(r)
            if r in eos_ids or n_tok >= stop_len:
                done = True
                break
        if stats is not None:
            stats.emitted += len(emitted)
        if on_round is not None:
            on_round({"k": k, "L": n_acc, "boundary": boundary, "emitted": emitted, "ids": ids, "preds": list(preds)})
        if done:
            return n_tok
        if drafter is not None:
            drafter.push([a for a in (atom_of(r, byte_offset, boundary_offset) for r in emitted) if a is not None])
        raw = emitted[-1]
        state, sub = automaton.step(states[n_acc], raw)
