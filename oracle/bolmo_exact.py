"""Float64 oracle of the batch-1 byte decoder -- TEST INFRASTRUCTURE ONLY.

The same model and loop as oracle/bolmo_ref.py (the Bolmo-shaped decoder of byteprof_b200.optim.bolmo_e2e:
byteprof/optim/bolmo_loop.py:182-207 for the loop, byteprof/optim/bolmo.py:32-136 for the layer and global
steps), with every activation kept in float64 and nothing rounded to bf16 or fp32: the value exact
arithmetic on the model's weights approaches. The weights are the model's bf16 values (exact in float64);
the rotary tables are the model's fp32 tables. The mLSTM step is the library formulation of
byteprof/optim/mlstm_multistep.py:20-86 (exponential gating with the max stabiliser) in float64.

BolmoDecoder(precision="fp32") runs the same model with fp32 activations; its greedy bytes and patch
decisions are checked against this oracle's.

Parity unpinned against the reference itself: Bolmo's model code is not part of byteprof, so no reference
output exists for this model; its pieces are pinned elsewhere (the skinny GEMM and the mLSTM recurrence
against the reference's golden vectors).
"""

from __future__ import annotations

import numpy as np

from .bolmo_ref import rope_tables

F64 = np.float64


def _f(a) -> np.ndarray:
    return np.asarray(a, dtype=F64)


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = _f(x)
    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * _f(w)


def sigmoid(x) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-_f(x)))


def swiglu(gu) -> np.ndarray:
    gu = _f(gu)
    ffn = gu.shape[-1] // 2
    g, u = gu[..., :ffn], gu[..., ffn:]
    return g * sigmoid(g) * u


def rope(x, cos, sin) -> np.ndarray:
    h = x.shape[-1] // 2
    a, b = x[:, :h], x[:, h:]
    return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)


class Attention:
    def __init__(self, nh: int, hd: int, max_pos: int):
        self.nh, self.hd = nh, hd
        self.k = np.zeros((max_pos, nh, hd), F64)
        self.v = np.zeros((max_pos, nh, hd), F64)

    def __call__(self, qkv, q_w, k_w, cos, sin, p: int, eps: float) -> np.ndarray:
        nh, hd = self.nh, self.hd
        d = nh * hd
        qkv = _f(qkv).reshape(-1)
        q = rmsnorm(qkv[None, :d], q_w, eps)[0].reshape(nh, hd)
        k = rmsnorm(qkv[None, d:2 * d], k_w, eps)[0].reshape(nh, hd)
        self.k[p] = rope(k, cos[p], sin[p])
        self.v[p] = qkv[2 * d:].reshape(nh, hd)
        s = np.einsum("hd,phd->hp", rope(q, cos[p], sin[p]), self.k[:p + 1]) * hd ** -0.5
        e = np.exp(s - s.max(axis=1, keepdims=True))
        o = np.einsum("hp,phd->hd", e, self.v[:p + 1]) / e.sum(axis=1, keepdims=True)
        return o.reshape(1, d)


def mlstm_step(state, q, k, v, i, f, qk_scale: float, eps: float):
    """One position for all heads in float64: (h [NH, DV], new state (C, n, m))."""
    c, n, m = state
    f_log = np.log(sigmoid(f))
    m_new = np.maximum(f_log + m, i)
    f_act = np.exp(f_log + m - m_new)
    i_act = np.exp(i - m_new)
    c = f_act[:, None, None] * c + i_act[:, None, None] * (k[:, :, None] * v[:, None, :])
    n = f_act[:, None] * n + i_act[:, None] * k
    qs = q * qk_scale
    num = np.einsum("hd,hde->he", qs, c)
    den = np.maximum(np.abs((qs * n).sum(axis=1)), np.exp(-m_new)) + eps
    return num / den[:, None], (c, n, m_new)


class LocalLayer:
    def __init__(self, wt: dict, prefix: str, nh: int, dh: int, cap: float = 15.0, eps: float = 1e-6,
                 mlstm_eps: float = 1e-6):
        self.w = {a: _f(wt[f"{prefix}.{a}"]) for a in ("norm1", "w_qkvo", "w_if", "b_if", "mh_norm", "w_out",
                                                       "norm2", "w_gu", "w_down")}
        self.nh, self.dh, self.cap, self.eps, self.mlstm_eps = nh, dh, cap, eps, mlstm_eps
        self.reset()

    def reset(self) -> None:
        nh, dh = self.nh, self.dh
        self.state = (np.zeros((nh, dh, dh), F64), np.zeros((nh, dh), F64), np.zeros(nh, F64))

    def step(self, h, x, out_norm):
        w, nh, dh, eps = self.w, self.nh, self.dh, self.eps
        d = nh * dh
        y = x @ w["w_qkvo"].T
        g = self.cap * np.tanh((x @ w["w_if"].T + w["b_if"]) / self.cap)
        q, k, v = (y[0, j * d:(j + 1) * d].reshape(nh, dh) for j in range(3))
        hs, self.state = mlstm_step(self.state, q, k, v, g[0, :nh], g[0, nh:], dh ** -0.5, self.mlstm_eps)
        z = sigmoid(y[:, 3 * d:]) * np.stack([rmsnorm(hs[j], w["mh_norm"][j], eps) for j in range(nh)]).reshape(1, d)
        h2 = h + z @ w["w_out"].T
        x2 = rmsnorm(h2, w["norm2"], eps)
        out = h2 + swiglu(x2 @ w["w_gu"].T) @ w["w_down"].T
        return rmsnorm(out, out_norm, eps)


class BolmoExact:
    """The whole decoder in float64: `feed(byte, new_patch)` returns (logits [vocab], boundary flag,
    boundary logit)."""

    def __init__(self, wt: dict, d: int = 2048, local_heads: int = 4, local_dh: int = 512, global_layers: int = 16,
                 global_heads: int = 16, max_patches: int = 1024, rope_theta: float = 500000.0, eps: float = 1e-6):
        self.wt = {k: _f(v) for k, v in wt.items()}
        self.d, self.eps, self.nl = d, eps, global_layers
        self.enc = LocalLayer(self.wt, "enc", local_heads, local_dh, eps=eps)
        self.dec = LocalLayer(self.wt, "dec", local_heads, local_dh, eps=eps)
        hd = d // global_heads
        cos, sin = rope_tables(max_patches, hd, rope_theta)  # the model's fp32 tables
        self.cos, self.sin = _f(cos), _f(sin)
        self.attn = [Attention(global_heads, hd, max_patches) for _ in range(global_layers)]
        self.reset()

    def reset(self) -> None:
        self.enc.reset()
        self.dec.reset()
        for a in self.attn:
            a.k[:] = 0.0
            a.v[:] = 0.0
        self.pos = 0
        self.value = np.zeros((1, self.d), F64)

    def glob(self, x) -> np.ndarray:
        w, eps = self.wt, self.eps
        for i in range(self.nl):
            g = f"glob{i}."
            att = self.attn[i](x @ w[g + "w_qkv"].T, w[g + "q_norm"], w[g + "k_norm"], self.cos, self.sin, self.pos,
                               eps)
            h = x + rmsnorm(att @ w[g + "w_o"].T, w[g + "attn_norm"], eps)
            x = h + rmsnorm(swiglu(h @ w[g + "w_gu"].T) @ w[g + "w_down"].T, w[g + "mlp_norm"], eps)
        self.pos += 1
        return x

    def feed(self, b: int, new_patch: bool) -> tuple[np.ndarray, bool, float]:
        w, eps = self.wt, self.eps
        h = w["embed"][b][None, :]
        e = self.enc.step(h, rmsnorm(h, self.enc.w["norm1"], eps), w["enc_norm"])
        bl = float((e @ w["w_boundary"].T)[0, 0])
        if new_patch:
            self.value = rmsnorm(self.glob(e @ w["w_patch"].T), w["dec_in_norm"], eps)
        hd = e @ w["w_in"].T + self.value
        xf = self.dec.step(hd, rmsnorm(hd, self.dec.w["norm1"], eps), w["final_norm"])
        logits = (xf @ w["lm_head"].T)[0]
        return logits, bool(sigmoid(bl) >= 0.5), bl


def greedy(model: BolmoExact, prompt: list[int], n_new: int) -> tuple[list[int], list[bool], list[float]]:
    """Greedy decoding as BolmoDecoder.generate: (generated bytes, whether each fed byte opened a patch, the
    top-2 logit gap of every step that chose a generated byte)."""
    new_patch, opened, tok, gaps = True, [], 0, []
    for b in prompt:
        opened.append(new_patch)
        logits, new_patch, _ = model.feed(b, new_patch)
        tok = int(np.argmax(logits))
    gaps.append(top2_gap(logits))
    out = []
    for i in range(n_new):
        out.append(tok)
        if i + 1 < n_new:
            opened.append(new_patch)
            logits, new_patch, _ = model.feed(tok, new_patch)
            tok = int(np.argmax(logits))
            gaps.append(top2_gap(logits))
    return out, opened, gaps


def top2_gap(logits) -> float:
    s = np.sort(_f(logits))
    return float(s[-1] - s[-2])
