"""The fp32-activation forms of the decoder's kernels (the exactness mode of BolmoDecoder) against the float64
oracle (oracle/bolmo_exact.py): the skinny linear reading x as fp32 (bf16 and int8 weights), RMSNorm in all
its fused modes, SwiGLU and the single-position attention with fp32 caches. Each result must be the float64
value to fp32 rounding of its sums: elementwise within REL of the largest magnitude (normwise), far below
one bf16 step."""

import numpy as np
import pytest
import torch

from byteprof_b200.optim import decode_ops as ops
from byteprof_b200.optim.skinny import skinny_mm
from helpers import deq_np, make_weights, randn, to_np
from oracle import bolmo_exact, bolmo_ref

pytestmark = pytest.mark.gpu
EPS = 1e-6
REL = 2e-6


def _near(a, b, rel=REL):
    a, b = np.asarray(to_np(a), np.float64), np.asarray(b, np.float64)
    err = float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
    assert err <= rel, err


def _f32(*shape, seed, scale=1.0):
    return randn(*shape, seed=seed, dtype=torch.float32, scale=scale)


@pytest.mark.parametrize("kind", ["bf16", "int8"])
@pytest.mark.parametrize("n,k", [(2048, 2048), (8192, 2048), (2048, 8192), (512, 2048), (1, 2048), (37, 264)])
def test_skinny_with_fp32_activations(kind, n, k):
    _, args = make_weights(kind, n, k, seed=5)
    x = _f32(4, k, seed=6)
    y = skinny_mm(x, *args, out=torch.empty(4, n, device="cuda"))
    w = deq_np(kind, args).astype(np.float64)
    ref = to_np(x).astype(np.float64) @ w.T
    bound = np.abs(to_np(x)).astype(np.float64) @ np.abs(w).T  # componentwise: |y - ref| / (|x| |W|)
    err = float((np.abs(to_np(y) - ref) / bound).max())
    assert err < 5e-6, err
    for m in (1, 2, 3):  # a row's bits do not depend on the other rows
        assert torch.equal(skinny_mm(x[:m].contiguous(), *args, out=torch.empty(m, n, device="cuda")), y[:m])


def test_skinny_fp32_activations_bf16_output_and_validation():
    _, (w,) = make_weights("bf16", 256, 512, seed=1)
    x = _f32(2, 512, seed=2)
    y = skinny_mm(x, w, out=torch.empty(2, 256, device="cuda", dtype=torch.bfloat16))
    yf = skinny_mm(x, w, out=torch.empty(2, 256, device="cuda"))
    assert torch.equal(y, yf.to(torch.bfloat16))
    assert skinny_mm(x, w).dtype == torch.float32  # the output follows x by default
    with pytest.raises(ValueError):
        skinny_mm(x.double(), w)


@pytest.mark.parametrize("rows,cols", [(1, 2048), (5, 512)])
def test_rmsnorm_modes_fp32(rows, cols):
    x, res = _f32(rows, cols, seed=3), _f32(rows, cols, seed=4, scale=3.0)
    w = randn(cols, seed=5, scale=0.1) + 1
    xs, rs, ws = (to_np(t).astype(np.float64) for t in (x, res, w))
    _near(ops.rmsnorm_ex(x, w, EPS), bolmo_exact.rmsnorm(xs, ws, EPS))
    h, n = ops.norm_add(x, res, w, EPS)
    _near(h, xs + rs, rel=1e-7)
    _near(n, bolmo_exact.rmsnorm(xs + rs, ws, EPS))
    _near(ops.add_norm(x, res, w, EPS), rs + bolmo_exact.rmsnorm(xs, ws, EPS))


def test_norm_gate_fp32():
    s, nh, dh = 2, 4, 512
    h = _f32(s, nh, dh, seed=12)
    o = _f32(s, nh * dh, seed=13)
    w = randn(nh, dh, seed=14, scale=0.1) + 1
    out = ops.norm_gate(h, o, w, EPS, torch.empty(s, nh * dh, device="cuda"))
    hs, os_, ws = (to_np(t).astype(np.float64) for t in (h, o, w))
    ref = bolmo_exact.sigmoid(os_) * np.stack([bolmo_exact.rmsnorm(hs[:, j], ws[j], EPS) for j in range(nh)],
                                             axis=1).reshape(s, nh * dh)
    _near(out, ref)


def test_swiglu_fp32():
    gu = _f32(3, 2 * 2816, seed=15, scale=2.0)
    _near(ops.swiglu(gu), bolmo_exact.swiglu(to_np(gu).astype(np.float64)))


def test_attention_fp32_over_a_growing_cache():
    nh, hd, max_pos = 16, 128, 1100
    d = nh * hd
    att = ops.DecodeAttention(nh, hd, max_pos, torch.device("cuda"), dtype=torch.float32)
    ref = bolmo_exact.Attention(nh, hd, max_pos)
    cos, sin = ops.rope_tables(max_pos, hd, 500000.0, torch.device("cuda"))
    rcos, rsin = (a.astype(np.float64) for a in bolmo_ref.rope_tables(max_pos, hd, 500000.0))
    qw, kw = randn(d, seed=1, scale=0.1) + 1, randn(d, seed=2, scale=0.1) + 1
    qws, kws = to_np(qw).astype(np.float64), to_np(kw).astype(np.float64)
    pos = torch.zeros(1, dtype=torch.long, device="cuda")
    for p in list(range(0, 40)) + [1023, 1024, 1099]:
        qkv = _f32(1, 3 * d, seed=100 + p)
        pos.fill_(p)
        out = att(qkv, qw, kw, cos, sin, pos, EPS)
        want = ref(to_np(qkv).astype(np.float64), qws, kws, rcos, rsin, p, EPS)
        _near(att.k_cache[p], ref.k[p])
        assert np.array_equal(to_np(att.v_cache[p]), ref.v[p].astype(np.float32))
        _near(out, want, rel=1e-5)  # softmax of scores that are themselves fp32 sums
