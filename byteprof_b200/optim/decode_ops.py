"""Fused glue operators of the batch-1 byte decoder, on the sm_100a kernels of csrc/decode.cu.

They replace the chains of small torch ops that byteprof's minimal Bolmo loop runs between its
GEMMs (byteprof/optim/bolmo.py:32-136, bolmo_loop.py:36-64):
  * embed_rmsnorm(t, i, w)   h = t[i], returns (h, rmsnorm(h) * w)             (byte embedding + first norm)
  * norm_add(x, res, w)      h = bf16(x + res), returns (h, rmsnorm(h) * w)   (pre-norm residual add)
  * add_norm(x, res, w)      res + rmsnorm(x) * w                              (OLMo-2 norm-after block)
  * norm_gate(h, o, w)       sigmoid(o) * rmsnorm(h) * w per head              (mLSTM output gate)
  * swiglu(gu)               silu(gate) * up
  * gate_softcap(g, b, cap)  cap * tanh((g + b) / cap), in place
  * DecodeAttention          one query position over a static KV cache (q/k RMSNorm, rotary
                             embedding, cache write, split attention)
  * decode_finish(logits, b, out)  out = [argmax(logits), sigmoid(b) >= 0.5]
  * GlobStep                 the whole global-model step (all OLMo-2 blocks) as one persistent kernel
  * LocStep                  the local encoder or decoder step (one mLSTM layer and its heads) as one
                             persistent kernel
Activations are bf16 or fp32 (one dtype per call; weights bf16). With bf16 every intermediate is rounded
where a bf16 torch tensor would hold it; with fp32 (the decoder's exactness mode) nothing is rounded to
bf16. CUDA tensors only; a missing library raises.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

NORM_PLAIN, NORM_ADD_FIRST, NORM_ADD_AFTER, NORM_GATE = 0, 1, 2, 3


def _bf16(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and t.dtype != torch.bfloat16:
            raise ValueError("bf16 tensors expected")


def _act(dtype: torch.dtype, *ts: torch.Tensor) -> int:
    """The C ABI code of the activation dtype (bf16 or fp32), which every given tensor must have."""
    if dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"activations must be bf16 or fp32, got {dtype}")
    for t in ts:
        if t is not None and t.dtype != dtype:
            raise ValueError(f"all activations of one call must be {dtype}")
    return _lib.dtype_code(dtype)


def _rows(t: torch.Tensor) -> tuple[int, int]:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("2-D tensors with unit column stride expected")
    return t.shape[0], t.stride(0)


def rmsnorm_ex(x: torch.Tensor, w: torch.Tensor, eps: float, mode: int = NORM_PLAIN, res: torch.Tensor | None = None,
               s_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """The general form on [rows, cols] bf16 or fp32 tensors with one bf16 weight row (w [cols])."""
    rows, ldx = _rows(x)
    cols = x.shape[1]
    y = out if out is not None else torch.empty(rows, cols, dtype=x.dtype, device=x.device)
    ldres = 0
    if res is not None:
        if res.shape[-1] != cols:
            raise ValueError("res must have cols columns")
        ldres = 0 if res.dim() == 1 or res.shape[0] == 1 else _rows(res)[1]
    lds = _rows(s_out)[1] if s_out is not None else 0
    _bf16(w)
    code = _act(x.dtype, res, s_out, y)
    if w.numel() != cols:
        raise ValueError("w must hold cols values")
    _lib.require_cuda(x, w, res, s_out, y)
    with _lib.on_device(x):
        _lib.call("bp_rmsnorm_ex", x.data_ptr(), ldx, w.data_ptr(), 1, _lib.ptr(res), ldres, _lib.ptr(s_out), lds,
                  y.data_ptr(), _rows(y)[1], rows, cols, eps, mode, code, _lib.stream_of(x))
    return y


def embed_rmsnorm(table: torch.Tensor, index: torch.Tensor, w: torch.Tensor, eps: float,
                  h_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(h, n) with h = table[index] (bf16 [rows, cols], index int64 [rows] on the device) and n = rmsnorm(h) * w,
    in one launch; an index outside the table gives NaN rows."""
    if index.dtype != torch.int64 or index.dim() != 1 or not index.is_contiguous():
        raise ValueError("index must be a contiguous int64 vector")
    rows, cols = index.numel(), table.shape[1]
    _, ldt = _rows(table)
    h = h_out if h_out is not None else torch.empty(rows, cols, dtype=table.dtype, device=table.device)
    y = out if out is not None else torch.empty(rows, cols, dtype=table.dtype, device=table.device)
    _bf16(table, w, h, y)
    if w.numel() != cols or h.shape != (rows, cols) or y.shape != (rows, cols):
        raise ValueError("w must hold cols values and h_out, out must be [rows, cols]")
    _lib.require_cuda(table, index, w, h, y)
    with _lib.on_device(table):
        _lib.call("bp_embed_rmsnorm", table.data_ptr(), ldt, table.shape[0], index.data_ptr(), w.data_ptr(),
                  h.data_ptr(), _rows(h)[1], y.data_ptr(), _rows(y)[1], rows, cols, eps, _lib.stream_of(table))
    return h, y


def norm_add(x: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float,
             want_sum: bool = True, out: torch.Tensor | None = None) -> tuple[torch.Tensor | None, torch.Tensor]:
    """(h, n) with h = x + res (rounded to x's dtype) and n = rmsnorm(h) * w; res may be one row (broadcast).
    n goes to `out` when given."""
    s = torch.empty_like(x) if want_sum else None
    return s, rmsnorm_ex(x, w, eps, NORM_ADD_FIRST, res=res, s_out=s, out=out)


def add_norm(x: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """res + rmsnorm(x) * w (with bf16: both roundings to bf16 as torch would do them)."""
    return rmsnorm_ex(x, w, eps, NORM_ADD_AFTER, res=res)


def norm_gate(h: torch.Tensor, o: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    """Per-head output gate of the mLSTM layer: h [S, NH, DH] (contiguous head rows), o [S, >= NH * DH]
    the o-gate pre-activations (row stride free), w [NH, DH]; out[s, j*DH:(j+1)*DH] = bf16(bf16(sigmoid(o))
    * rmsnorm(h[s, j]) * w[j])."""
    s, nh, dh = h.shape
    if h.stride(2) != 1 or h.stride(1) != dh or tuple(w.shape) != (nh, dh) or not w.is_contiguous():
        raise ValueError("h needs contiguous (NH, DH) rows and w must be a contiguous [NH, DH]")
    if o.stride(1) != 1 or out.stride(1) != 1 or o.shape[0] < s or out.shape[0] < s:
        raise ValueError("o and out need unit column strides and S rows")
    _bf16(w)
    code = _act(h.dtype, o, out)
    _lib.require_cuda(h, o, w, out)
    with _lib.on_device(h):
        _lib.call("bp_rmsnorm_ex", h.data_ptr(), h.stride(0), w.data_ptr(), nh, o.data_ptr(), o.stride(0), None, 0,
                  out.data_ptr(), out.stride(0), s * nh, dh, eps, NORM_GATE, code, _lib.stream_of(h))
    return out


def swiglu(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """gu [rows, 2 * ffn] (gate | up) -> silu(gate) * up [rows, ffn] (bf16: bf16(bf16(silu(gate)) * up))."""
    rows, ld = _rows(gu)
    ffn = gu.shape[1] // 2
    y = out if out is not None else torch.empty(rows, ffn, dtype=gu.dtype, device=gu.device)
    code = _act(gu.dtype, y)
    _lib.require_cuda(gu, y)
    with _lib.on_device(gu):
        _lib.call("bp_swiglu", gu.data_ptr(), ld, y.data_ptr(), _rows(y)[1], rows, ffn, code, _lib.stream_of(gu))
    return y


def gate_softcap(g: torch.Tensor, bias: torch.Tensor | None, cap: float) -> torch.Tensor:
    """In place on g [rows, n] fp32: g <- cap * tanh((g + bias) / cap)."""
    rows, ld = _rows(g)
    if g.dtype != torch.float32 or (bias is not None and (bias.dtype != torch.float32 or bias.numel() != g.shape[1])):
        raise ValueError("fp32 g and bias of n values expected")
    _lib.require_cuda(g, bias)
    with _lib.on_device(g):
        _lib.call("bp_gate_softcap", g.data_ptr(), ld, _lib.ptr(bias), g.data_ptr(), ld, rows, g.shape[1], cap,
                  _lib.stream_of(g))
    return g


def decode_finish(logits: torch.Tensor, boundary_logit: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
    """out[0] = argmax(logits) (torch order), out[1] = sigmoid(boundary_logit) >= 0.5; int64 out."""
    if logits.dtype != torch.float32 or not logits.is_contiguous() or out.dtype != torch.int64 or out.numel() < 2:
        raise ValueError("contiguous fp32 logits and an int64 out of >= 2 values expected")
    if boundary_logit is not None and boundary_logit.dtype != torch.float32:
        raise ValueError("fp32 boundary logit expected")
    _lib.require_cuda(logits, boundary_logit, out)
    with _lib.on_device(logits):
        _lib.call("bp_decode_finish", logits.data_ptr(), logits.numel(), _lib.ptr(boundary_logit), out.data_ptr(),
                  _lib.stream_of(logits))
    return out


def rope_tables(max_pos: int, head_dim: int, theta: float, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin [max_pos, head_dim / 2] fp32 of angle p * theta^(-2i / head_dim), computed in float64 on
    the host."""
    inv = 1.0 / theta ** (torch.arange(0, head_dim // 2, dtype=torch.float64) * 2 / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().to(device), torch.sin(ang).float().to(device)


class DecodeAttention:
    """Static KV caches of one layer and its single-position attention; activations and caches of `dtype`
    (bf16, or fp32 for the exactness mode)."""

    def __init__(self, nh: int, head_dim: int, max_pos: int, device: torch.device,
                 dtype: torch.dtype = torch.bfloat16):
        self.nh, self.hd, self.max_pos, self.dtype = nh, head_dim, max_pos, dtype
        self.k_cache = torch.zeros(max_pos, nh, head_dim, dtype=dtype, device=device)
        self.v_cache = torch.zeros(max_pos, nh, head_dim, dtype=dtype, device=device)

    def reset(self) -> None:
        self.k_cache.zero_()
        self.v_cache.zero_()

    def __call__(self, qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, cos: torch.Tensor,
                 sin: torch.Tensor, pos: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
        d = self.nh * self.hd
        if qkv.dtype != self.dtype or qkv.numel() != 3 * d or not qkv.is_contiguous():
            raise ValueError(f"qkv must be a contiguous {self.dtype} [1, 3 * nh * head_dim]")
        if pos.dtype != torch.int64 or cos.shape != (self.max_pos, self.hd // 2) or sin.shape != cos.shape:
            raise ValueError("int64 pos and cos / sin tables [max_pos, head_dim / 2] expected")
        y = out if out is not None else torch.empty(1, d, dtype=self.dtype, device=qkv.device)
        _bf16(q_norm, k_norm)
        code = _act(self.dtype, y)
        _lib.require_cuda(qkv, q_norm, k_norm, cos, sin, pos, y)
        with _lib.on_device(qkv):
            _lib.call("bp_decode_attention", qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(),
                      sin.data_ptr(), pos.data_ptr(), self.k_cache.data_ptr(), self.v_cache.data_ptr(), y.data_ptr(),
                      self.nh, self.hd, self.max_pos, eps, self.hd ** -0.5, code, _lib.stream_of(qkv))
        return y


class _GlobLayer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("w_qkv", "q_norm", "k_norm", "w_o", "attn_norm", "w_gu", "w_down",
                                               "mlp_norm", "k_cache", "v_cache")]


class GlobStep:
    """The global-model step of a Bolmo-1B-shaped decoder (OLMo-2 blocks of d 2048, 16 heads x 128, SwiGLU
    8192) in one persistent kernel (bp_glob_step): value = rmsnorm(blocks(x)) * out_norm at patch position
    *pos, which it advances by one. `blocks` are objects with the attributes w_qkv, q_norm, k_norm, w_o,
    attn_norm, w_gu, w_down, mlp_norm and attn (a DecodeAttention holding the caches)."""

    def __init__(self, blocks, out_norm: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, max_pos: int,
                 eps: float):
        self.keep = list(blocks)  # the tensors must outlive every launch (and graph) that uses them
        self.layers = (_GlobLayer * len(blocks))()
        for i, b in enumerate(blocks):
            ts = (b.w_qkv, b.q_norm, b.k_norm, b.w_o, b.attn_norm, b.w_gu, b.w_down, b.mlp_norm, b.attn.k_cache,
                  b.attn.v_cache)
            for t in ts:
                if t.dtype != torch.bfloat16 or not t.is_contiguous() or not t.is_cuda:
                    raise ValueError("global-step weights and caches must be contiguous bf16 CUDA tensors")
            self.layers[i] = _GlobLayer(*(t.data_ptr() for t in ts))
        self.out_norm, self.cos, self.sin, self.max_pos, self.eps = out_norm, cos, sin, max_pos, eps
        dev = out_norm.device
        # zero-filled once: it carries the kernel's launch number from one launch to the next
        self.workspace = torch.zeros(int(_lib.lib().bp_glob_step_workspace_bytes()), dtype=torch.uint8, device=dev)

    def __call__(self, x: torch.Tensor, value_out: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        _bf16(x, value_out)
        if pos.dtype != torch.int64:
            raise ValueError("pos must be a device int64")
        _lib.require_cuda(x, value_out, pos)
        with _lib.on_device(x):
            _lib.call("bp_glob_step", ctypes.addressof(self.layers), len(self.keep), x.data_ptr(),
                      self.out_norm.data_ptr(), value_out.data_ptr(), pos.data_ptr(), self.cos.data_ptr(),
                      self.sin.data_ptr(), self.max_pos, self.eps, self.workspace.data_ptr(), self.workspace.numel(),
                      _lib.stream_of(x))
        return value_out


class _LocLayer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("norm1", "w_qkvo", "w_if", "b_if", "mh_norm", "w_out", "norm2", "w_gu",
                                               "w_down", "c", "n_cur", "m_cur", "n_next", "m_next")]


class LocStep:
    """One local step of a Bolmo-shaped decoder (one mLSTM layer of d 2048, 4 heads x 512, SwiGLU 2816, and
    the encoder's patch / boundary heads or the decoder's LM head and argmax) as one persistent kernel
    (bp_loc_enc_step / bp_loc_dec_step). `layer` is a bolmo_local.LocalLayer; `parity` names the n / m
    buffers holding the current state, as in LocalLayer.step."""

    def __init__(self, layer):
        self.layer = layer
        c = layer.state[0]
        w = (layer.norm1, layer.w_qkvo, layer.w_if, layer.b_if, layer.mh_norm, layer.w_out, layer.norm2, layer.w_gu,
             layer.w_down)
        for t in (*w, c, *layer.nm[0], *layer.nm[1]):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError("local-step weights and state must be contiguous CUDA tensors")
        self.tables = []
        for parity in (0, 1):
            n_cur, m_cur = layer.nm[parity]
            n_next, m_next = layer.nm[1 - parity]
            self.tables.append(_LocLayer(*(t.data_ptr() for t in w), c.data_ptr(), n_cur.data_ptr(), m_cur.data_ptr(),
                                         n_next.data_ptr(), m_next.data_ptr()))
        # zero-filled once: it carries the kernel's launch number from one launch to the next
        self.workspace = torch.zeros(int(_lib.lib().bp_loc_step_workspace_bytes()), dtype=torch.uint8, device=c.device)

    def _common(self, parity: int):
        layer = self.layer
        return (layer.norm_eps, layer.gate_cap, layer.mlstm_eps, self.workspace.data_ptr(), self.workspace.numel(),
                _lib.stream_of(self.workspace))

    def enc(self, parity: int, embed, byte, enc_norm, w_patch, w_boundary, e_out, patch_out, boundary_logit) -> None:
        with _lib.on_device(embed):
            _lib.call("bp_loc_enc_step", ctypes.addressof(self.tables[parity]), embed.data_ptr(), byte.data_ptr(),
                      enc_norm.data_ptr(), w_patch.data_ptr(), w_boundary.data_ptr(), e_out.data_ptr(),
                      patch_out.data_ptr(), boundary_logit.data_ptr(), *self._common(parity))

    def encdec(self, dec: "LocStep", parity: int, embed, byte, enc_norm, w_patch, w_boundary, e_out, patch_out,
               boundary_logit, value, w_in, final_norm, lm_head, logits, out) -> None:
        """This (encoder) step and then `dec`'s decoder step of the same byte in one launch
        (bp_loc_encdec_step), for a byte that opens no patch; this step's workspace."""
        a, b = self.layer, dec.layer
        if (a.norm_eps, a.gate_cap, a.mlstm_eps) != (b.norm_eps, b.gate_cap, b.mlstm_eps):
            raise ValueError("the fused local step needs the encoder and decoder layers' eps and gate cap to agree")
        with _lib.on_device(embed):
            _lib.call("bp_loc_encdec_step", ctypes.addressof(self.tables[parity]), ctypes.addressof(dec.tables[parity]),
                      embed.data_ptr(), byte.data_ptr(), enc_norm.data_ptr(), w_patch.data_ptr(), w_boundary.data_ptr(),
                      e_out.data_ptr(), patch_out.data_ptr(), boundary_logit.data_ptr(), value.data_ptr(),
                      w_in.data_ptr(), final_norm.data_ptr(), lm_head.data_ptr(), logits.data_ptr(), out.data_ptr(),
                      *self._common(parity))

    def dec(self, parity: int, e_in, value, w_in, final_norm, lm_head, boundary_logit, logits, out) -> None:
        with _lib.on_device(e_in):
            _lib.call("bp_loc_dec_step", ctypes.addressof(self.tables[parity]), e_in.data_ptr(), value.data_ptr(),
                      w_in.data_ptr(), final_norm.data_ptr(), lm_head.data_ptr(), boundary_logit.data_ptr(),
                      logits.data_ptr(), out.data_ptr(), *self._common(parity))
