"""The decoder's fused glue kernels (csrc/decode.cu) against the numpy oracle (oracle/bolmo_ref.py):
RMSNorm with its residual add / norm-after add / output gate, SwiGLU, the gate soft cap, the split
single-position attention with q/k RMSNorm, rotary embedding and the cache write, and the argmax +
boundary finish. bf16 results: within one bf16 step of the oracle everywhere and equal to it in
>= 99 % of elements (the oracle sums in another order, so a rounding can land one step apart)."""

import numpy as np
import pytest
import torch

from byteprof_b200.optim import decode_ops as ops
from byteprof_b200.optim.bolmo_local import rmsnorm
from helpers import bf16_step_close, randn, to_np
from oracle import bolmo_ref

pytestmark = pytest.mark.gpu
EPS = 1e-6


def _close(a, b, min_exact=0.99):
    ok, worst, exact = bf16_step_close(to_np(a), np.asarray(b, np.float32), min_exact)
    assert ok, (worst, exact)


@pytest.mark.parametrize("rows,cols", [(1, 2048), (5, 2048), (33, 512), (3, 8)])
def test_plain_mode_is_bp_rmsnorm_bit_for_bit(rows, cols):
    x = randn(rows, cols, seed=1)
    w = randn(cols, seed=2, scale=0.1) + 1
    y = ops.rmsnorm_ex(x, w, EPS)
    assert torch.equal(y, rmsnorm(x, w, EPS))
    _close(y, bolmo_ref.rmsnorm(to_np(x), to_np(w), EPS))


@pytest.mark.parametrize("rows,cols", [(1, 2048), (3, 2048), (2, 10240)])
def test_embed_rmsnorm_is_gather_then_norm(rows, cols):
    table = randn(512, cols, seed=21)
    w = randn(cols, seed=22, scale=0.1) + 1
    idx = torch.tensor([7, 511, 0][:rows], dtype=torch.long, device="cuda")
    h, y = ops.embed_rmsnorm(table, idx, w, EPS)
    g = table.index_select(0, idx)
    assert torch.equal(h, g)
    assert torch.equal(y, ops.rmsnorm_ex(g, w, EPS))  # the same kernel and order as the plain norm
    _close(y, bolmo_ref.rmsnorm(to_np(g), to_np(w), EPS))


def test_embed_rmsnorm_index_outside_the_table_gives_nan_rows():
    table = randn(16, 2048, seed=23)
    w = randn(2048, seed=24, scale=0.1) + 1
    idx = torch.tensor([3, 16, -1], dtype=torch.long, device="cuda")
    h, y = ops.embed_rmsnorm(table, idx, w, EPS)
    assert torch.equal(h[0], table[3])
    assert torch.isnan(h[1:]).all() and torch.isnan(y[1:]).all()
    assert not torch.isnan(y[0]).any()


@pytest.mark.parametrize("rows", [1, 7])
def test_norm_add_against_the_oracle(rows):
    x, res = randn(rows, 2048, seed=3), randn(rows, 2048, seed=4, scale=3.0)
    w = randn(2048, seed=5, scale=0.1) + 1
    h, n = ops.norm_add(x, res, w, EPS)
    rh, rn = bolmo_ref.norm_add(to_np(x), to_np(res), to_np(w), EPS)
    assert np.array_equal(to_np(h), rh)  # a bf16 sum of two bf16 values: exact
    _close(n, rn)
    assert torch.equal(n, rmsnorm(h, w, EPS))  # the same row order as bp_rmsnorm


def test_norm_add_broadcasts_a_single_residual_row():
    x, res = randn(4, 2048, seed=6), randn(1, 2048, seed=7)
    w = randn(2048, seed=8, scale=0.1) + 1
    h, n = ops.norm_add(x, res, w, EPS)
    for r in range(4):
        h1, n1 = ops.norm_add(x[r:r + 1], res, w, EPS)
        assert torch.equal(h1, h[r:r + 1]) and torch.equal(n1, n[r:r + 1])


def test_add_norm_against_the_oracle_with_strided_rows():
    big = randn(6, 4096, seed=9)
    x = big[:, 1024:3072]  # row stride 4096
    res = randn(6, 2048, seed=10, scale=2.0)
    w = randn(2048, seed=11, scale=0.1) + 1
    y = ops.add_norm(x, res, w, EPS)
    _close(y, bolmo_ref.add_norm(to_np(x), to_np(res), to_np(w), EPS))


@pytest.mark.parametrize("s", [1, 9])
def test_norm_gate_per_head_against_the_oracle(s):
    nh, dh = 4, 512
    h = randn(s, nh, dh, seed=12)
    y = randn(s, 4 * nh * dh, seed=13)
    o = y[:, 3 * nh * dh:]  # the o-gate columns of a [S, 4d] projection
    w = randn(nh, dh, seed=14, scale=0.1) + 1
    out = torch.empty(s, nh * dh, dtype=torch.bfloat16, device="cuda")
    ops.norm_gate(h, o, w, EPS, out)
    _close(out, bolmo_ref.norm_gate(to_np(h), to_np(o), to_np(w), EPS))


@pytest.mark.parametrize("rows,ffn", [(1, 8192), (3, 2816), (2, 8)])
def test_swiglu_against_the_oracle(rows, ffn):
    gu = randn(rows, 2 * ffn, seed=15, scale=2.0)
    _close(ops.swiglu(gu), bolmo_ref.swiglu(to_np(gu)), min_exact=0.999)


def test_gate_softcap_against_the_oracle():
    g = randn(5, 8, seed=16, dtype=torch.float32, scale=20.0)
    b = torch.tensor([0.0] * 4 + [3.0] * 4, device="cuda")
    ref = bolmo_ref.gate_softcap(to_np(g), to_np(b), 15.0)
    out = ops.gate_softcap(g.clone(), b, 15.0)
    np.testing.assert_allclose(to_np(out), ref, rtol=2e-6, atol=1e-6)


def test_norm_validation():
    x = randn(2, 2048, seed=1)
    w = randn(2048, seed=2)
    with pytest.raises(ValueError):
        ops.rmsnorm_ex(x, w[:100], EPS)
    with pytest.raises(Exception):  # misaligned column count reaches the C checks
        ops.rmsnorm_ex(randn(2, 12, seed=3), randn(12, seed=4), EPS)


class _Attn:
    """Random q | k | v per position through the kernel and the oracle side by side."""

    def __init__(self, nh=16, hd=128, max_pos=1024, seed=0):
        self.nh, self.hd, self.d = nh, hd, nh * hd
        self.k = ops.DecodeAttention(nh, hd, max_pos, torch.device("cuda"))
        self.ref = bolmo_ref.Attention(nh, hd, max_pos)
        self.cos, self.sin = ops.rope_tables(max_pos, hd, 500000.0, torch.device("cuda"))
        self.rcos, self.rsin = bolmo_ref.rope_tables(max_pos, hd, 500000.0)
        self.qw = randn(self.d, seed=seed + 1, scale=0.1) + 1
        self.kw = randn(self.d, seed=seed + 2, scale=0.1) + 1
        self.pos = torch.zeros(1, dtype=torch.long, device="cuda")
        self.seed = seed

    def step(self, p):
        """One position through both; the oracle then attends over the kernel's own cache row of p (the
        two compute k with sums in another order, so a k value can round one bf16 step apart, which
        moves the softmax by a little; the cache rows are compared separately)."""
        qkv = randn(1, 3 * self.d, seed=1000 * self.seed + p)
        self.pos.fill_(p)
        out = self.k(qkv, self.qw, self.kw, self.cos, self.sin, self.pos, EPS)
        self.ref(to_np(qkv), to_np(self.qw), to_np(self.kw), self.rcos, self.rsin, p, EPS)
        kc, rk = to_np(self.k.k_cache[p]), self.ref.k[p].copy()
        assert np.mean(kc == rk) > 0.99 and np.abs(kc - rk).max() <= 2.0**-7 * np.abs(rk).max(), p
        assert np.array_equal(to_np(self.k.v_cache[p]), self.ref.v[p]), p
        self.ref.k[p] = kc
        return out, self.ref.attend(to_np(qkv), to_np(self.qw), self.rcos, self.rsin, p, EPS)


def _attn_close(out, ref):
    """Normwise within a bf16 step of the largest output, and >= 95 % of elements equal to the oracle
    rounded to bf16 (q is normalised in another summation order, so a q value can round one step apart)."""
    from oracle.bf16 import round_bf16

    o = to_np(out)
    err = float(np.abs(o - ref).max() / np.abs(ref).max())
    exact = float(np.mean(o == round_bf16(ref)))
    return err <= 2.0**-8 and exact >= 0.95, err, exact


def test_attention_over_a_growing_cache_against_the_oracle():
    a = _Attn()
    for p in range(0, 200):
        out, ref = a.step(p)
        ok, err, exact = _attn_close(out, ref)
        assert ok, (p, err, exact)


@pytest.mark.parametrize("max_pos,positions", [(1024, (700, 1023)), (2500, (1024, 1100, 2047, 2048, 2499))])
def test_attention_many_chunks_rounds_and_the_last_position(max_pos, positions):
    """Every CTA of the cluster busy, and caches longer than one 1024-position round (the running
    softmax rescaled between rounds)."""
    a = _Attn(seed=3, max_pos=max_pos)
    g = torch.Generator(device="cuda").manual_seed(9)
    fill = (torch.randn(max_pos, a.nh, a.hd, generator=g, device="cuda")).to(torch.bfloat16)
    a.k.k_cache.copy_(fill)
    a.k.v_cache.copy_(fill.flip(0))
    a.ref.k[:] = to_np(fill)
    a.ref.v[:] = to_np(fill.flip(0))
    for p in positions:
        out, ref = a.step(p)
        ok, err, exact = _attn_close(out, ref)
        assert ok, (p, err, exact)


def test_attention_graph_replays_follow_the_device_position():
    a = _Attn(seed=5)
    qkv = randn(1, 3 * a.d, seed=77)
    out = torch.empty(1, a.d, dtype=torch.bfloat16, device="cuda")
    a.pos.fill_(0)
    a.k(qkv, a.qw, a.kw, a.cos, a.sin, a.pos, EPS, out=out)  # warm-up outside capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        a.k(qkv, a.qw, a.kw, a.cos, a.sin, a.pos, EPS, out=out)
    eager = ops.DecodeAttention(a.nh, a.hd, 1024, torch.device("cuda"))
    for p in (0, 1, 64, 65, 300):
        a.pos.fill_(p)
        g.replay()
        e = eager(qkv, a.qw, a.kw, a.cos, a.sin, a.pos, EPS)
        assert torch.equal(out, e), p
    torch.cuda.synchronize()


def test_attention_rejects_a_position_outside_the_cache_without_writing():
    a = _Attn(seed=7)
    a.pos.fill_(5000)
    qkv = randn(1, 3 * a.d, seed=5)
    out = a.k(qkv, a.qw, a.kw, a.cos, a.sin, a.pos, EPS)
    assert torch.isnan(out.float()).all()
    assert int(a.k.k_cache.abs().sum()) == 0 and int(a.k.v_cache.abs().sum()) == 0


def test_finish_argmax_order_and_boundary_flag():
    out = torch.zeros(2, dtype=torch.long, device="cuda")
    for n in (1, 512, 1000):
        x = randn(n, seed=n, dtype=torch.float32)
        for b in (-0.3, 0.0, 2.0):
            ops.decode_finish(x, torch.tensor([b], device="cuda"), out)
            assert int(out[0]) == int(torch.argmax(x)) and int(out[1]) == int(torch.sigmoid(torch.tensor(b)) >= 0.5)
    x = torch.zeros(512, device="cuda")
    x[[7, 300]] = 5.0  # ties: lowest index
    ops.decode_finish(x, None, out)
    assert out.tolist() == [7, 0]
    x[400] = float("nan")  # NaN is the largest, as torch.argmax
    ops.decode_finish(x, None, out)
    assert int(out[0]) == 400 == int(torch.argmax(x))
