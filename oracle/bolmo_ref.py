"""Oracle for the batch-1 byte decoder (numpy, CPU) -- TEST INFRASTRUCTURE ONLY.

A restatement of the Bolmo-shaped decoder of byteprof_b200.optim.bolmo_e2e at the rounding points of
its kernels, rebuilt from the model's weights (`BolmoDecoder.weights()` as float32 arrays):
  * the minimal decode loop: byteprof/optim/bolmo_loop.py:182-207 (per byte: encoder step, the global
    step when the previous step flagged a boundary, decoder step, argmax) and the static-KV global step
    of byteprof/optim/bolmo.py:100-136;
  * the local layer step: byteprof/optim/bolmo.py:32-44 with the Bolmo-shaped mLSTM layer (the
    recurrence is `mlstm_ref.step` in its bf16 precision model, mlstm_multistep.py:20-86);
  * the glue: RMSNorm (with its residual add, the OLMo-2 norm-after add, the per-head output gate),
    SwiGLU, the gate soft cap, single-position attention with q/k RMSNorm and rotary embedding, the
    argmax and the boundary test.
Every value a bf16 tensor holds on the GPU is rounded to bf16 here at the same point; arithmetic in
between is float32 (matrix products: float32 BLAS over exact bf16 x bf16 products; softmax and
transcendentals in float64, then rounded). Sums are taken in a different order than the kernels', so
the two agree to float32 rounding, and a bf16 rounding of an intermediate can land one step apart.

Parity unpinned against the reference itself: Bolmo's model code is not part of byteprof, so no
reference output exists for this model; the pieces it is built from are pinned elsewhere (the skinny
GEMM and the mLSTM recurrence against the reference's golden vectors).
"""

from __future__ import annotations

import numpy as np

from . import mlstm_ref
from .bf16 import round_bf16

F32 = np.float32
F64 = np.float64


def _f32(a) -> np.ndarray:
    return np.asarray(a, dtype=F32)


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """bf16(x * (1 / sqrt(mean(x^2) + eps)) * w) row-wise, x [rows, cols]; the mean, the sum, the square
    root and the reciprocal each rounded to float32 as the kernels do (the sum of squares is exact here,
    the kernels' is an fp32 sum)."""
    x = _f32(x)
    ss = (x.astype(F64) ** 2).sum(axis=-1, keepdims=True).astype(F32)
    t = ((ss / F32(x.shape[-1])).astype(F32) + F32(eps)).astype(F32)
    inv = (F32(1.0) / np.sqrt(t)).astype(F32)
    return round_bf16((x * inv).astype(F32) * _f32(w))


def norm_add(x, res, w, eps: float):
    """(h, n): h = bf16(x + res), n = rmsnorm(h) * w."""
    h = round_bf16(_f32(x) + _f32(res))
    return h, rmsnorm(h, w, eps)


def add_norm(x, res, w, eps: float) -> np.ndarray:
    """bf16(res + rmsnorm(x) * w)."""
    return round_bf16(_f32(res) + rmsnorm(x, w, eps))


def sigmoid(x) -> np.ndarray:
    return (1.0 / (1.0 + np.exp(-_f32(x).astype(F64)))).astype(F32)


def norm_gate(h, o, w, eps: float) -> np.ndarray:
    """h [S, NH, DH], o [S, NH * DH], w [NH, DH] -> bf16(bf16(sigmoid(o)) * rmsnorm(h[s, j]) * w[j])."""
    s, nh, dh = h.shape
    n = np.stack([rmsnorm(h[:, j], w[j], eps) for j in range(nh)], axis=1).reshape(s, nh * dh)
    return round_bf16(round_bf16(sigmoid(o)) * n)


def swiglu(gu) -> np.ndarray:
    gu = _f32(gu)
    ffn = gu.shape[-1] // 2
    g, u = gu[..., :ffn], gu[..., ffn:]
    silu = round_bf16((g.astype(F64) / (1.0 + np.exp(-g.astype(F64)))).astype(F32))
    return round_bf16(silu * u)


def gate_softcap(g, bias, cap: float) -> np.ndarray:
    t = (_f32(g) + _f32(bias)).astype(F32)
    return (F32(cap) * np.tanh((t / F32(cap)).astype(F32).astype(F64)).astype(F32)).astype(F32)


def linear(x, w, bf16_out: bool = True) -> np.ndarray:
    """x [M, K] @ w[N, K]^T in float32 (the products of bf16 values are exact), optionally rounded to bf16."""
    y = (_f32(x) @ _f32(w).T).astype(F32)
    return round_bf16(y) if bf16_out else y


def rope_tables(max_pos: int, hd: int, theta: float):
    inv = 1.0 / theta ** (np.arange(0, hd // 2, dtype=F64) * 2 / hd)
    ang = np.arange(max_pos, dtype=F64)[:, None] * inv[None, :]
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rope(x, cos, sin) -> np.ndarray:
    """Rotary halves of x [NH, HD] in float32: (a c - b s, b c + a s)."""
    h = x.shape[-1] // 2
    a, b = x[:, :h], x[:, h:]
    return np.concatenate([(a * cos).astype(F32) - (b * sin).astype(F32),
                           (b * cos).astype(F32) + (a * sin).astype(F32)], axis=-1).astype(F32)


class Attention:
    """Static KV cache of one OLMo-2 layer and the single-position attention of bp_decode_attention."""

    def __init__(self, nh: int, hd: int, max_pos: int):
        self.nh, self.hd = nh, hd
        self.k = np.zeros((max_pos, nh, hd), F32)
        self.v = np.zeros((max_pos, nh, hd), F32)

    def __call__(self, qkv, q_w, k_w, cos, sin, p: int, eps: float) -> np.ndarray:
        """Writes k, v of position p into the cache, then attends over positions 0..p."""
        nh, hd = self.nh, self.hd
        d = nh * hd
        qkv = _f32(qkv).reshape(-1)
        k = rmsnorm(qkv[None, d:2 * d], k_w, eps)[0].reshape(nh, hd)
        self.k[p] = round_bf16(rope(k, cos[p], sin[p]))
        self.v[p] = qkv[2 * d:].reshape(nh, hd)
        return self.attend(qkv, q_w, cos, sin, p, eps)

    def attend(self, qkv, q_w, cos, sin, p: int, eps: float) -> np.ndarray:
        """The attention of position p's query over the cache as it stands (positions 0..p)."""
        nh, hd = self.nh, self.hd
        d = nh * hd
        qkv = _f32(qkv).reshape(-1)
        q = rmsnorm(qkv[None, :d], q_w, eps)[0].reshape(nh, hd)
        qr = rope(q, cos[p], sin[p])
        scale = F32(hd ** -0.5)
        s = np.einsum("hd,phd->hp", qr.astype(F64), self.k[:p + 1].astype(F64)).astype(F32) * scale
        s = s.astype(F64)
        e = np.exp(s - s.max(axis=1, keepdims=True))
        o = np.einsum("hp,phd->hd", e, self.v[:p + 1].astype(F64)) / e.sum(axis=1, keepdims=True)
        return round_bf16(o.astype(F32)).reshape(1, d)


class LocalLayer:
    """The Bolmo-shaped mLSTM layer, one position per step (state advances)."""

    def __init__(self, wt: dict, prefix: str, nh: int, dh: int, ffn: int, cap: float = 15.0, eps: float = 1e-6,
                 mlstm_eps: float = 1e-6):
        self.w = {a: _f32(wt[f"{prefix}.{a}"]) for a in ("norm1", "w_qkvo", "w_if", "b_if", "mh_norm", "w_out",
                                                         "norm2", "w_gu", "w_down")}
        self.nh, self.dh, self.ffn, self.cap, self.eps, self.mlstm_eps = nh, dh, ffn, cap, eps, mlstm_eps
        self.reset()

    def reset(self) -> None:
        nh, dh = self.nh, self.dh
        self.state = (np.zeros((nh, dh, dh), F32), np.zeros((nh, dh), F32), np.zeros(nh, F32))

    def step(self, h, x, out_norm=None):
        """h, x [1, d] (x = rmsnorm(h) * norm1) -> (h_out, rmsnorm(h_out) * out_norm or None)."""
        w, nh, dh = self.w, self.nh, self.dh
        d = nh * dh
        y = linear(x, w["w_qkvo"])
        g = gate_softcap(linear(x, w["w_if"], bf16_out=False), w["b_if"], self.cap)
        q, k, v = (y[0, j * d:(j + 1) * d].reshape(nh, dh) for j in range(3))
        hs, self.state = mlstm_ref.step(self.state, q, k, v, g[0, :nh], g[0, nh:], dh ** -0.5, self.mlstm_eps,
                                        bf16=True)
        self.last = {"x": x, "y": y, "g": g, "h": hs}  # intermediates, for diagnostics
        z = norm_gate(hs[None], y[:, 3 * d:], w["mh_norm"], self.eps)
        h2, x2 = norm_add(linear(z, w["w_out"]), h, w["norm2"], self.eps)
        dn = linear(swiglu(linear(x2, w["w_gu"])), w["w_down"])
        if out_norm is None:
            return round_bf16(h2 + dn), None
        return norm_add(dn, h2, out_norm, self.eps)


class BolmoRef:
    """The whole decoder on the CPU: `feed(byte, new_patch)` returns (logits [vocab] fp32, boundary flag)."""

    def __init__(self, wt: dict, d: int = 2048, vocab: int = 512, local_heads: int = 4, local_dh: int = 512,
                 local_ffn: int = 2816, global_layers: int = 16, global_heads: int = 16, max_patches: int = 1024,
                 rope_theta: float = 500000.0, eps: float = 1e-6):
        self.wt = {k: _f32(v) for k, v in wt.items()}
        self.d, self.vocab, self.eps, self.nl = d, vocab, eps, global_layers
        self.enc = LocalLayer(self.wt, "enc", local_heads, local_dh, local_ffn, eps=eps)
        self.dec = LocalLayer(self.wt, "dec", local_heads, local_dh, local_ffn, eps=eps)
        hd = d // global_heads
        self.cos, self.sin = rope_tables(max_patches, hd, rope_theta)
        self.attn = [Attention(global_heads, hd, max_patches) for _ in range(global_layers)]
        self.reset()

    def reset(self) -> None:
        self.enc.reset()
        self.dec.reset()
        self.pos = 0
        self.value = np.zeros((1, self.d), F32)

    def glob(self, patch) -> np.ndarray:
        w, eps, x = self.wt, self.eps, patch
        for i in range(self.nl):
            g = f"glob{i}."
            att = self.attn[i](linear(x, w[g + "w_qkv"]), w[g + "q_norm"], w[g + "k_norm"], self.cos, self.sin,
                               self.pos, eps)
            h = add_norm(linear(att, w[g + "w_o"]), x, w[g + "attn_norm"], eps)
            dn = linear(swiglu(linear(h, w[g + "w_gu"])), w[g + "w_down"])
            x = add_norm(dn, h, w[g + "mlp_norm"], eps)
        self.pos += 1
        return x

    def feed(self, b: int, new_patch: bool) -> tuple[np.ndarray, bool, float]:
        """One byte. Returns (logits [vocab] fp32, boundary flag, boundary logit)."""
        w, eps = self.wt, self.eps
        h = w["embed"][b][None, :]
        _, e = self.enc.step(h, rmsnorm(h, self.enc.w["norm1"], eps), out_norm=w["enc_norm"])
        bl = linear(e, w["w_boundary"], bf16_out=False)[0, 0]
        if new_patch:
            self.value = rmsnorm(self.glob(linear(e, w["w_patch"])), w["dec_in_norm"], eps)
        hd, x = norm_add(linear(e, w["w_in"]), self.value, self.dec.w["norm1"], eps)
        _, xf = self.dec.step(hd, x, out_norm=w["final_norm"])
        logits = linear(xf, w["lm_head"], bf16_out=False)[0]
        self.last = {"e": e, "value": self.value, "xf": xf}  # intermediates, for diagnostics
        return logits, bool(sigmoid(bl) >= F32(0.5)), float(bl)


def greedy(model: BolmoRef, prompt: list[int], n_new: int) -> tuple[list[int], list[bool]]:
    """Greedy decoding as BolmoDecoder.generate: (generated bytes, whether each fed byte opened a patch)."""
    new_patch, opened, tok = True, [], 0
    for b in prompt:
        opened.append(new_patch)
        logits, new_patch, _ = model.feed(b, new_patch)
        tok = int(np.argmax(logits))
    out = []
    for i in range(n_new):
        out.append(tok)
        if i + 1 < n_new:
            opened.append(new_patch)
            logits, new_patch, _ = model.feed(tok, new_patch)
            tok = int(np.argmax(logits))
    return out, opened


def top2_gap(logits) -> float:
    s = np.sort(_f32(logits))
    return float(s[-1] - s[-2])
