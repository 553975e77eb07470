"""A Bolmo-shaped local (byte-level) model on the sm_100a kernels, and its drafting verify round.

Mirrors the fused verification of byteprof/optim/bolmo_draft.py:29-135 (`DraftEngine` with
verify="fused"): the local encoder and decoder run over the S = K + 1 positions of a round, every
projection a skinny GEMM over the S rows, the mLSTM recurrence the fused multi-position scan
(`multistep_fw`, the state left untouched); the logits' argmax, the draft acceptance and the lazy state
commit (positions 0..L, L read on the device) close the round, and each S is one CUDA graph, so a round
costs one host synchronisation whatever L turns out to be.

Bolmo's remote model code is not part of byteprof, so the model here is random-initialised with
Bolmo-1B's local shapes, one mLSTM layer each for the encoder and the decoder:
  * byte embedding 512 x d; decoder input = in_projection(encoder output) + the last global patch
    vector (a fixed random vector here: the global model is not part of the verify round);
  * layer (bolmo_draft.py:74-100): RMSNorm -> q, k, v, o-gate pre-activation (one [4d, d] skinny GEMM)
    and input / forget gate pre-activations ([2 NH, d], fp32 out, forget bias +3, soft cap 15) ->
    fused scan over NH heads of dim dh -> per-head RMSNorm -> sigmoid(o) * h -> out_proj -> residual
    -> RMSNorm -> SwiGLU MLP (width 2816: gate and up as one [2 * 2816, d] GEMM, down [d, 2816]) ->
    residual;
  * final RMSNorm and LM head 512 x d; greedy argmax.
The steps between the GEMMs (RMSNorm with its residual add, the per-head output gate, SwiGLU, the gate
soft cap) are the fused kernels of `decode_ops`. Every step is row-independent (the skinny kernels' K partition depends on (N, K) only, the norms sum
each row in a fixed order, the scan computes position t the same way for any number of positions), so
a round that verifies K correct drafts yields the bits of K + 1 single-position rounds.
"""

from __future__ import annotations

import torch

from .. import _lib
from . import draft_fused
from .decode_ops import NORM_PLAIN, gate_softcap, norm_add, norm_gate, rmsnorm_ex, swiglu
from .draft_core import mlstm_scan
from .skinny import skinny_mm


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-wise RMSNorm of a bf16 [rows, cols] tensor (rows may be strided) on the sm_100a kernel; an fp32 x
    (the exactness mode) gives an fp32 result through the same kernel family."""
    if x.dtype == torch.float32:
        return rmsnorm_ex(x, w, eps, NORM_PLAIN, out=out)
    rows, cols = x.shape
    y = out if out is not None else torch.empty(rows, cols, dtype=torch.bfloat16, device=x.device)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise ValueError("rmsnorm takes bf16 x, w and out")
    if x.stride(1) != 1 or y.stride(1) != 1 or w.numel() != cols:
        raise ValueError("rmsnorm needs unit column strides and w of cols entries")
    _lib.require_cuda(x, w, y)
    with _lib.on_device(x):
        _lib.call("bp_rmsnorm", x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), rows, cols, eps,
                  _lib.stream_of(x))
    return y


class LocalLayer:
    """One Bolmo-shaped mLSTM block with its recurrent state (c, n, m).

    `forward` runs S positions for a verify round (the state is read, not changed; `commit` applies
    positions 0..L later). `step` runs one position of the decode loop and advances the state: c is
    updated in place, n and m alternate between two buffers (the scan's CTAs all read n and m, so they
    cannot be written in place); `parity` names the buffer holding the current n and m.
    """

    def __init__(self, d: int, nh: int, dh: int, ffn: int, gen: torch.Generator, device: torch.device,
                 smax: int, std: float = 0.02, gate_cap: float = 15.0, norm_eps: float = 1e-6,
                 mlstm_eps: float = 1e-6, act_dtype: torch.dtype = torch.bfloat16):
        def rnd(*shape, scale=std):
            return (torch.randn(*shape, generator=gen, device=device) * scale).to(torch.bfloat16)

        self.d, self.nh, self.dh, self.ffn, self.act = d, nh, dh, ffn, act_dtype
        self.gate_cap, self.norm_eps, self.mlstm_eps = gate_cap, norm_eps, mlstm_eps
        self.norm1 = (1.0 + rnd(d)).to(torch.bfloat16)
        self.w_qkvo = rnd(4 * d, d)
        self.w_if = rnd(2 * nh, d)
        self.b_if = torch.cat([torch.zeros(nh), torch.full((nh,), 3.0)]).to(device)  # input 0, forget +3
        self.mh_norm = (1.0 + rnd(nh, dh)).to(torch.bfloat16)
        self.w_out = rnd(d, d)
        self.norm2 = (1.0 + rnd(d)).to(torch.bfloat16)
        self.w_gu = rnd(2 * ffn, d)
        self.w_down = rnd(d, ffn)
        f32 = dict(dtype=torch.float32, device=device)
        self.state = (torch.zeros(1, nh, dh, dh, **f32), torch.zeros(1, nh, dh, **f32), torch.zeros(1, nh, 1, **f32))
        self.nm = ((self.state[1], self.state[2]), (torch.zeros(1, nh, dh, **f32), torch.zeros(1, nh, 1, **f32)))
        self.nstart = torch.zeros(nh, dh, **f32)
        self.mstart = torch.zeros(nh, **f32)
        self.hbuf = torch.zeros(smax, nh, dh, dtype=act_dtype, device=device)
        self.saved: dict[int, tuple[torch.Tensor, ...]] = {}

    def reset(self) -> None:
        for t in (*self.state, *self.nm[1]):
            t.zero_()

    def current_state(self, parity: int = 0) -> tuple[torch.Tensor, ...]:
        return (self.state[0], *self.nm[parity])

    def _project(self, x: torch.Tensor):
        s, d, nh, dh = x.shape[0], self.d, self.nh, self.dh
        y = skinny_mm(x, self.w_qkvo)  # [S, 4d]: q | k | v | o
        g = skinny_mm(x, self.w_if, out=torch.empty(s, 2 * nh, dtype=torch.float32, device=x.device))
        gate_softcap(g, self.b_if, self.gate_cap)
        q, k, v = (y[:, j * d:(j + 1) * d].view(s, nh, dh) for j in range(3))
        return y, q, k, v, g[:, :nh].reshape(s, nh, 1), g[:, nh:].reshape(s, nh, 1)

    def _tail(self, h: torch.Tensor, y: torch.Tensor, s: int, out_norm: torch.Tensor | None, want_sum: bool,
              out: torch.Tensor | None = None):
        d, eps = self.d, self.norm_eps
        z = norm_gate(self.hbuf[:s], y[:, 3 * d:], self.mh_norm, eps,
                      out=torch.empty(s, d, dtype=self.act, device=h.device))
        h2, x2 = norm_add(skinny_mm(z, self.w_out), h, self.norm2, eps)
        dn = skinny_mm(swiglu(skinny_mm(x2, self.w_gu)), self.w_down)
        if out_norm is None:
            return h2 + dn, None
        return norm_add(dn, h2, out_norm, eps, want_sum, out=out)

    def forward(self, h: torch.Tensor, x: torch.Tensor | None = None, out_norm: torch.Tensor | None = None,
                want_sum: bool = True):
        """h [S, d] bf16 (contiguous) -> (h_out [S, d], rmsnorm(h_out) * out_norm or None). x is
        rmsnorm(h) * norm1 when the caller has it already (fused with the add that made h). The state is
        read, not changed (see `commit`)."""
        s = h.shape[0]
        if x is None:
            x = rmsnorm(h, self.norm1, self.norm_eps)
        y, q, k, v, i_pre, f_pre = self._project(x)
        draft_fused.multistep_fw(self.state, q, k, v, i_pre, f_pre, self.hbuf, self.nstart, self.mstart,
                                 eps=self.mlstm_eps)
        self.saved[s] = (k, v, i_pre, f_pre)
        return self._tail(h, y, s, out_norm, want_sum)

    def commit(self, length: torch.Tensor, s: int) -> None:
        """state <- the state after positions 0..L of the last S-position forward (L on the device)."""
        k, v, i_pre, f_pre = self.saved[s]
        draft_fused.lazy_commit(self.state, k, v, i_pre, f_pre, length, self.nstart, self.mstart)

    def step(self, h: torch.Tensor, x: torch.Tensor, parity: int, out_norm: torch.Tensor | None = None,
             want_sum: bool = True, out: torch.Tensor | None = None):
        """One position ([1, d]) of the decode loop; the state advances (n, m from buffer `parity` to
        buffer 1 - parity). Returns as `forward` (the normalised output into `out` when given)."""
        y, q, k, v, i_pre, f_pre = self._project(x)
        mlstm_scan(self.current_state(parity), q, k, v, i_pre, f_pre, self.hbuf, self.current_state(1 - parity),
                   self.mlstm_eps)
        return self._tail(h, y, 1, out_norm, want_sum, out)


class BolmoLocal:
    """Encoder layer + decoder layer + LM head of a Bolmo-shaped byte model, with graphed verify rounds."""

    def __init__(self, device: torch.device | str = "cuda", seed: int = 0, d: int = 2048, nh: int = 4,
                 dh: int = 512, ffn: int = 2816, vocab: int = 512, smax: int = 33):
        device = torch.device(device)
        gen = torch.Generator(device=device).manual_seed(seed)
        self.device, self.d, self.vocab, self.smax = device, d, vocab, smax
        self.embed = (torch.randn(vocab, d, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.enc = LocalLayer(d, nh, dh, ffn, gen, device, smax)
        self.dec = LocalLayer(d, nh, dh, ffn, gen, device, smax)
        self.w_in = (torch.randn(d, d, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.last_value = torch.randn(d, generator=gen, device=device).to(torch.bfloat16)
        self.final_norm = (1.0 + torch.randn(d, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.lm_head = (torch.randn(vocab, d, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.ids = torch.zeros(smax, dtype=torch.long, device=device)
        self.tok = torch.zeros(smax, dtype=torch.long, device=device)
        self.out = torch.zeros(smax + 1, dtype=torch.long, device=device)  # [tok_0 .. tok_{S-1}, ..., L]
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._pin_ids = torch.zeros(smax, dtype=torch.long).pin_memory()
        self._pin_out = torch.zeros(smax + 1, dtype=torch.long).pin_memory()

    def reset(self) -> None:
        self.enc.reset()
        self.dec.reset()

    def round(self, s: int) -> None:
        """One verify round over ids[:s] on the device: tokens, acceptance and the state commit."""
        h, _ = self.enc.forward(self.embed.index_select(0, self.ids[:s]))
        hd, x = norm_add(skinny_mm(h, self.w_in), self.last_value, self.dec.norm1, self.dec.norm_eps)
        _, xf = self.dec.forward(hd, x, out_norm=self.final_norm, want_sum=False)
        logits = skinny_mm(xf, self.lm_head, out=torch.empty(s, self.vocab, dtype=torch.float32, device=self.device))
        self.tok[:s].copy_(torch.argmax(logits, dim=-1))
        draft_fused.accept(self.ids, self.tok, self.out, s, self.smax)
        length = self.out[self.smax:]
        self.enc.commit(length, s)
        self.dec.commit(length, s)

    def capture(self, ks: tuple[int, ...]) -> None:
        """One CUDA graph per K (S = K + 1). Warm-up runs go through the same buffers; the state is
        saved around them, so capturing does not advance the model."""
        saved = [t.clone() for layer in (self.enc, self.dec) for t in layer.state]
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_):
            for k in ks:
                self.round(k + 1)
        torch.cuda.current_stream().wait_stream(s_)
        for k in ks:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.round(k + 1)
            self.graphs[k + 1] = g
        torch.cuda.synchronize()
        for dst, src in zip([t for layer in (self.enc, self.dec) for t in layer.state], saved):
            dst.copy_(src)

    def verify(self, ids: list[int]) -> tuple[list[int], int]:
        """Run the round for ids = [last byte, draft_1, ..., draft_K] (graph if captured): returns the
        predicted tokens and the accepted length L; the state advances by positions 0..L."""
        s = len(ids)
        if not 1 <= s <= self.smax:
            raise ValueError(f"a round holds 1..{self.smax} positions")
        self._pin_ids[:s] = torch.tensor(ids, dtype=torch.long)
        self.ids[:s].copy_(self._pin_ids[:s], non_blocking=True)
        g = self.graphs.get(s)
        if g is not None:
            g.replay()
        else:
            self.round(s)
        self._pin_out.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        out = self._pin_out.tolist()
        return out[:s], out[self.smax]
