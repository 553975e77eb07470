"""The decoder oracle (oracle/bolmo_ref.py) on its own, on the CPU: its attention against a plain float64
softmax attention with the rotary embedding written out independently, its glue against the formulas,
and the greedy loop of a tiny random model (structure and determinism)."""

import numpy as np

from oracle import bolmo_ref
from oracle.bf16 import round_bf16


def _bf(rng, *shape, scale=1.0):
    return round_bf16(rng.standard_normal(shape).astype(np.float32) * scale)


def test_attention_against_a_float64_restatement():
    rng = np.random.default_rng(0)
    nh, hd, maxp, eps = 4, 128, 80, 1e-6
    d = nh * hd
    att = bolmo_ref.Attention(nh, hd, maxp)
    cos, sin = bolmo_ref.rope_tables(maxp, hd, 500000.0)
    qw, kw = 1 + _bf(rng, d, scale=0.05), 1 + _bf(rng, d, scale=0.05)
    ks, vs = [], []
    for p in range(70):
        qkv = _bf(rng, 3 * d)
        out = att(qkv, qw, kw, cos, sin, p, eps)

        def norm(x, w):
            x = x.astype(np.float64)
            return round_bf16((x / np.sqrt((x * x).mean() + eps) * w).astype(np.float32)).astype(np.float64)

        def rot(x):
            ang = p * 500000.0 ** (-np.arange(hd // 2) * 2 / hd)
            a, b = x[:, :hd // 2], x[:, hd // 2:]
            return np.concatenate([a * np.cos(ang) - b * np.sin(ang), b * np.cos(ang) + a * np.sin(ang)], axis=1)

        q = rot(norm(qkv[:d], qw).reshape(nh, hd))
        ks.append(round_bf16(rot(norm(qkv[d:2 * d], kw).reshape(nh, hd)).astype(np.float32)).astype(np.float64))
        vs.append(qkv[2 * d:].reshape(nh, hd).astype(np.float64))
        s = np.einsum("hd,phd->hp", q, np.stack(ks)) / np.sqrt(hd)
        pr = np.exp(s - s.max(1, keepdims=True))
        ref = np.einsum("hp,phd->hd", pr / pr.sum(1, keepdims=True), np.stack(vs)).reshape(1, d)
        assert np.abs(out - ref).max() <= 2.0**-7 * np.abs(ref).max() + 1e-6, p


def test_glue_formulas():
    rng = np.random.default_rng(1)
    x, res, w = _bf(rng, 3, 64), _bf(rng, 3, 64, scale=2), 1 + _bf(rng, 64, scale=0.1)
    n = bolmo_ref.rmsnorm(x, w, 1e-6)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 ** 2).mean(1, keepdims=True) + 1e-6) * w
    assert np.abs(n - ref).max() <= 2.0**-7 * np.abs(ref).max()
    h, n2 = bolmo_ref.norm_add(x, res, w, 1e-6)
    assert np.array_equal(h, round_bf16(x + res)) and np.array_equal(n2, bolmo_ref.rmsnorm(h, w, 1e-6))
    assert np.array_equal(bolmo_ref.add_norm(x, res, w, 1e-6), round_bf16(res + n))
    gu = _bf(rng, 2, 16, scale=3)
    g, u = gu[:, :8].astype(np.float64), gu[:, 8:].astype(np.float64)
    assert np.abs(bolmo_ref.swiglu(gu) - g / (1 + np.exp(-g)) * u).max() <= 2.0**-6 * np.abs(g * u).max()
    cap = bolmo_ref.gate_softcap(np.array([[100.0, -100.0, 0.0]], np.float32), np.zeros(3, np.float32), 15.0)
    assert np.allclose(cap, [[15.0, -15.0, 0.0]], atol=1e-5)


def _tiny_weights(seed, d=64, nh=2, dh=32, ffn=96, gl=2, gffn=128, vocab=512):
    rng = np.random.default_rng(seed)
    w = {"embed": _bf(rng, vocab, d, scale=0.5), "enc_norm": 1 + _bf(rng, d, scale=0.02),
         "w_boundary": _bf(rng, 1, d, scale=0.2), "w_patch": _bf(rng, d, d, scale=0.1),
         "dec_in_norm": 1 + _bf(rng, d, scale=0.02), "w_in": _bf(rng, d, d, scale=0.1),
         "final_norm": 1 + _bf(rng, d, scale=0.02), "lm_head": _bf(rng, vocab, d, scale=0.2)}
    for p in ("enc", "dec"):
        w.update({f"{p}.norm1": 1 + _bf(rng, d, scale=0.02), f"{p}.w_qkvo": _bf(rng, 4 * d, d, scale=0.1),
                  f"{p}.w_if": _bf(rng, 2 * nh, d, scale=0.1), f"{p}.b_if": np.array([0.0] * nh + [3.0] * nh, np.float32),
                  f"{p}.mh_norm": 1 + _bf(rng, nh, dh, scale=0.02), f"{p}.w_out": _bf(rng, d, d, scale=0.1),
                  f"{p}.norm2": 1 + _bf(rng, d, scale=0.02), f"{p}.w_gu": _bf(rng, 2 * ffn, d, scale=0.1),
                  f"{p}.w_down": _bf(rng, d, ffn, scale=0.1)})
    for i in range(gl):
        g = f"glob{i}."
        w.update({g + "w_qkv": _bf(rng, 3 * d, d, scale=0.1), g + "q_norm": 1 + _bf(rng, d, scale=0.02),
                  g + "k_norm": 1 + _bf(rng, d, scale=0.02), g + "w_o": _bf(rng, d, d, scale=0.1),
                  g + "attn_norm": 1 + _bf(rng, d, scale=0.02), g + "w_gu": _bf(rng, 2 * gffn, d, scale=0.1),
                  g + "w_down": _bf(rng, d, gffn, scale=0.1), g + "mlp_norm": 1 + _bf(rng, d, scale=0.02)})
    return w


def test_tiny_model_greedy_loop():
    kw = dict(d=64, local_heads=2, local_dh=32, local_ffn=96, global_layers=2, global_heads=2, max_patches=64)
    m = bolmo_ref.BolmoRef(_tiny_weights(3), **kw)
    prompt = [5, 17, 200, 3, 99]
    gen, opened = bolmo_ref.greedy(m, prompt, 12)
    assert len(gen) == 12 and len(opened) == len(prompt) + 11 and opened[0]
    assert all(0 <= t < 512 for t in gen)
    assert 1 <= m.pos == sum(opened) <= len(opened)
    m.reset()
    assert bolmo_ref.greedy(m, prompt, 12) == (gen, opened)  # deterministic from a reset
    # teacher forcing with its own tokens reproduces the same logits' argmax at every step
    m.reset()
    fed, new_patch = prompt + gen[:-1], True
    toks = []
    for b in fed:
        logits, new_patch, _ = m.feed(b, new_patch)
        toks.append(int(np.argmax(logits)))
    assert toks[len(prompt) - 1:] == gen
