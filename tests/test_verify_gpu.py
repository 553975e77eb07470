"""The drafting verify path on a Bolmo-shaped local model (byteprof_b200.optim.bolmo_local), following
the reference's drafting contract (byteprof/optim/bolmo_draft.py:1-8, draft_core.py): verifying K drafts
in one round must give exactly what K + 1 single-position rounds give. Checked bit for bit (tokens,
accepted length, the committed encoder and decoder states), for all-correct drafts and for a wrong draft
at every position; the CUDA-graph rounds against eager ones with the accepted length changing between
replays; the row-wise RMSNorm against fp32 and for row independence; and one local layer against a plain
PyTorch fp32 restatement of the same block (the scan through the numpy oracle)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from byteprof_b200.optim.bolmo_local import BolmoLocal, LocalLayer, rmsnorm
from helpers import to_np
from oracle import mlstm_ref

pytestmark = pytest.mark.gpu


def _states(model):
    return [t.clone() for layer in (model.enc, model.dec) for t in layer.state]


def _same(a, b):
    return all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.fixture(scope="module")
def model():
    return BolmoLocal(seed=3)


@pytest.fixture(scope="module")
def sequential(model):
    """Greedy single-position rounds from byte 65: the tokens and the states after each step."""
    model.reset()
    cur, toks, states = 65, [], []
    for _ in range(34):
        t, n = model.verify([cur])
        assert n == 0
        toks.append(t[0])
        states.append(_states(model))
        cur = t[0]
    return toks, states


def test_rmsnorm_matches_fp32_and_rows_are_independent():
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(33, 2048, generator=g, device="cuda").to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(2048, generator=g, device="cuda")).to(torch.bfloat16)
    y = rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert ((y.float() - ref).abs() <= ref.abs() * 2.0**-7 + 1e-6).all()
    for r in (0, 5, 16, 32):
        assert torch.equal(rmsnorm(x[r:r + 1], w, 1e-6), y[r:r + 1])


@pytest.mark.parametrize("k", [1, 4, 15, 32])
def test_correct_drafts_give_the_sequential_result_bit_for_bit(model, sequential, k):
    toks, states = sequential
    model.reset()
    t, n = model.verify([65] + toks[:k])
    assert n == k and t == toks[:k + 1]
    assert _same(_states(model), states[k])


@pytest.mark.parametrize("j", [0, 1, 3, 7])
def test_a_wrong_draft_stops_acceptance_there(model, sequential, j):
    toks, states = sequential
    k = 8
    drafts = list(toks[:k])
    drafts[j] = (drafts[j] + 1) % 512
    model.reset()
    t, n = model.verify([65] + drafts)
    assert n == j and t[:j + 1] == toks[:j + 1]
    assert _same(_states(model), states[j])


def test_graphed_rounds_equal_eager_ones_with_a_changing_length(sequential):
    toks, states = sequential
    m = BolmoLocal(seed=3)
    m.capture((0, 4, 8))
    assert set(m.graphs) == {1, 5, 9}
    m.reset()
    t, n = m.verify([65] + toks[:8])           # all 8 accepted
    assert n == 8 and t == toks[:9] and _same(_states(m), states[8])
    bad = list(toks[9:13])
    bad[2] = (bad[2] + 7) % 512
    t, n = m.verify([toks[8]] + bad)            # same graph size 5, now 2 accepted
    assert n == 2 and t[:3] == toks[9:12] and _same(_states(m), states[11])
    t, n = m.verify([toks[11]])                 # the single-position graph
    assert n == 0 and t == [toks[12]] and _same(_states(m), states[12])


def test_one_layer_against_an_fp32_restatement():
    torch.manual_seed(0)
    gen = torch.Generator(device="cuda").manual_seed(5)
    layer = LocalLayer(2048, 4, 512, 2816, gen, torch.device("cuda"), smax=9)
    h = (torch.randn(9, 2048, generator=gen, device="cuda")).to(torch.bfloat16)
    out = layer.forward(h)[0].float()

    def norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()

    hf = h.float()
    x = norm(hf, layer.norm1)
    y = x @ layer.w_qkvo.float().T
    g = 15.0 * torch.tanh((x @ layer.w_if.float().T + layer.b_if) / 15.0)
    d, nh, dh = 2048, 4, 512
    q, k, v = (to_np(y[:, j * d:(j + 1) * d]).reshape(9, nh, dh) for j in range(3))
    state = (np.zeros((nh, dh, dh), np.float32), np.zeros((nh, dh), np.float32), np.zeros(nh, np.float32))
    hs, _, _ = mlstm_ref.multistep_fw(state, q, k, v, to_np(g[:, :nh]), to_np(g[:, nh:]), dh ** -0.5, 1e-6,
                                      bf16=False)
    hs = torch.from_numpy(np.ascontiguousarray(hs)).to("cuda")
    hn = torch.cat([norm(hs[:, j], layer.mh_norm[j]) for j in range(nh)], dim=-1)
    h2 = hf + (torch.sigmoid(y[:, 3 * d:]) * hn) @ layer.w_out.float().T
    gu = norm(h2, layer.norm2) @ layer.w_gu.float().T
    ref = h2 + (F.silu(gu[:, :2816]) * gu[:, 2816:]) @ layer.w_down.float().T
    rel = float((out - ref).norm() / ref.norm())
    assert rel < 2e-2, rel  # bf16 activations between the kernels against an all-fp32 restatement
