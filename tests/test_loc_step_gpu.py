"""The local encoder and decoder steps as one persistent kernel each (bp_loc_enc_step / bp_loc_dec_step,
csrc/loc_step.cu) against the same steps kernel by kernel (LocalLayer.step with the skinny GEMMs, the scan
and the decode.cu glue), from the same weights and recurrent state. The two differ in summation orders
(CUDA-core dot products against tensor-core tiles, the mLSTM unit's sums), so a bf16 rounding lands one step
apart now and then and the layer's noise-dominated heads spread it; the outputs and the new state stay
within a few percent normwise and strongly correlated. Also: CUDA-graph replays equal eager launches, and a
byte outside the vocabulary writes NaN and leaves the state alone."""

import numpy as np
import pytest
import torch

from byteprof_b200.optim.bolmo_e2e import BolmoDecoder
from helpers import to_np

pytestmark = pytest.mark.gpu


def _model(seed=7):
    m = BolmoDecoder(seed=seed, global_layers=1, fused_local=True)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    for layer in (m.enc, m.dec):  # a non-trivial recurrent state
        c, n, mm = layer.state
        c.copy_(torch.randn(c.shape, generator=g, device="cuda") * 0.05)
        n.copy_(torch.randn(n.shape, generator=g, device="cuda") * 0.5)
        mm.copy_(torch.randn(mm.shape, generator=g, device="cuda"))
    m.value.copy_(torch.randn(m.value.shape, generator=g, device="cuda").to(torch.bfloat16))
    m.e.copy_(torch.randn(m.e.shape, generator=g, device="cuda").to(torch.bfloat16))
    return m


def _snap(layer):
    return [t.clone() for t in (*layer.state, *layer.nm[1])]


def _restore(layer, snap):
    for t, v in zip((*layer.state, *layer.nm[1]), snap):
        t.copy_(v)


def _np(t):
    return to_np(t) if torch.is_tensor(t) else np.asarray(t)


def _stats(a, b):
    a, b = _np(a).ravel().astype(np.float64), _np(b).ravel().astype(np.float64)
    err = float(np.abs(a - b).max() / np.abs(b).max())
    corr = float(np.corrcoef(a, b)[0, 1])
    return err, corr


def _run(m, which, fused):
    kern = m.enc_kernel if which == "enc" else m.dec_kernel
    if which == "enc":
        m.enc_kernel = kern if fused else None
        m.enc_step(0)
        m.enc_kernel = kern
    else:
        m.dec_kernel = kern if fused else None
        m.dec_step(0)
        m.dec_kernel = kern
    torch.cuda.synchronize()


@pytest.mark.parametrize("byte", [0, 65, 255, 511])
def test_encoder_step_matches_the_kernel_by_kernel_step(byte):
    m = _model()
    snap = _snap(m.enc)
    m.byte.fill_(byte)
    _run(m, "enc", fused=False)
    ref = [m.e.clone(), m.patch.clone(), m.boundary_logit.clone(), m.enc.state[0].clone(), m.enc.nm[1][0].clone(),
           m.enc.nm[1][1].clone()]
    _restore(m.enc, snap)
    _run(m, "enc", fused=True)
    got = [m.e, m.patch, m.boundary_logit, m.enc.state[0], m.enc.nm[1][0], m.enc.nm[1][1]]
    names = ["e", "patch", "boundary", "C", "n", "m"]
    stats = {nm: _stats(g, r) for nm, g, r in zip(names, got, ref) if nm != "boundary"}
    stats["boundary"] = float(abs(float(got[2]) - float(ref[2])))
    print(byte, stats)
    for nm in ("e", "patch"):
        assert stats[nm][0] <= 0.05 and stats[nm][1] >= 0.995, (nm, stats[nm])
    for nm in ("C", "n"):
        assert stats[nm][0] <= 0.02 and stats[nm][1] >= 0.9999, (nm, stats[nm])
    assert stats["m"][0] <= 1e-5, stats["m"]
    assert stats["boundary"] <= 0.05 * max(1.0, abs(float(ref[2])))
    # the current buffers were only read
    assert all(torch.equal(a, b) for a, b in zip((m.enc.nm[0][0], m.enc.nm[0][1]), (snap[1], snap[2])))


def test_decoder_step_matches_the_kernel_by_kernel_step():
    m = _model(11)
    snap = _snap(m.dec)
    m.boundary_logit.fill_(0.3)
    _run(m, "dec", fused=False)
    ref_logits, ref_state = m.logits.clone(), m.dec.state[0].clone()
    _restore(m.dec, snap)
    m.out.zero_()
    _run(m, "dec", fused=True)
    err, corr = _stats(m.logits, ref_logits)
    cerr, ccorr = _stats(m.dec.state[0], ref_state)
    print({"logits": (err, corr), "C": (cerr, ccorr)})
    assert err <= 0.05 and corr >= 0.995, (err, corr)
    assert cerr <= 0.02 and ccorr >= 0.9999, (cerr, ccorr)
    lg = m.logits.float()
    assert int(m.out[0]) == int(torch.argmax(lg)) and int(m.out[1]) == 1  # sigmoid(0.3) >= 0.5


def test_graph_replays_equal_eager_launches():
    m = _model(3)
    snap_e, snap_d = _snap(m.enc), _snap(m.dec)
    m.byte.fill_(42)
    m.enc_step(0)
    m.dec_step(0)
    eager = [m.e.clone(), m.patch.clone(), m.logits.clone(), m.out.clone(), m.enc.state[0].clone()]
    _restore(m.enc, snap_e)
    _restore(m.dec, snap_d)
    ge, gd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(ge):
        m.enc_step(0)
    with torch.cuda.graph(gd):
        m.dec_step(0)
    _restore(m.enc, snap_e)
    _restore(m.dec, snap_d)
    ge.replay()
    gd.replay()
    torch.cuda.synchronize()
    got = [m.e, m.patch, m.logits, m.out, m.enc.state[0]]
    assert all(torch.equal(a, b) for a, b in zip(got, eager))


def test_a_byte_outside_the_vocabulary_writes_nan_and_leaves_the_state():
    m = _model(5)
    snap = _snap(m.enc)
    m.byte.fill_(512)
    m.enc_step(0)
    torch.cuda.synchronize()
    assert torch.isnan(m.e.float()).all() and torch.isnan(m.patch.float()).all()
    assert torch.isnan(m.boundary_logit).all()
    assert all(torch.equal(a, b) for a, b in zip((*m.enc.state, *m.enc.nm[1]), snap))


def _oracle_layer(m, layer, name):
    from oracle import bolmo_ref
    w = {k: to_np(v) for k, v in m.weights().items()}
    ref = bolmo_ref.LocalLayer(w, name, layer.nh, layer.dh, layer.ffn)
    c, n, mm = layer.current_state(0)
    ref.state = (to_np(c[0]), to_np(n[0]), to_np(mm[0, :, 0]))
    return w, ref


@pytest.mark.parametrize("byte", [3, 200])
def test_both_encoder_steps_against_the_oracle(byte):
    """The persistent encoder step and the kernel-by-kernel one against the numpy oracle from the same weights
    and state: the persistent kernel is no farther from the oracle than the kernel-by-kernel step (both differ
    from it only in summation orders), on the outputs and on the new state."""
    from oracle import bolmo_ref
    m = _model(13)
    w, ref = _oracle_layer(m, m.enc, "enc")
    h = w["embed"][byte][None, :]
    _, e = ref.step(h, bolmo_ref.rmsnorm(h, ref.w["norm1"], 1e-6), out_norm=w["enc_norm"])
    want = {"e": e, "patch": bolmo_ref.linear(e, w["w_patch"]), "C": ref.state[0]}
    snap = _snap(m.enc)
    m.byte.fill_(byte)
    got = {}
    for fused in (False, True):
        _restore(m.enc, snap)
        _run(m, "enc", fused)
        got[fused] = {"e": m.e.clone(), "patch": m.patch.clone(), "C": m.enc.state[0][0].clone()}
    stats = {k: (_stats(got[False][k], want[k]), _stats(got[True][k], want[k])) for k in want}
    print(byte, stats)
    for k, ((e_kbk, c_kbk), (e_f, c_f)) in stats.items():
        assert e_f <= max(1.5 * e_kbk, 0.01) and c_f >= min(c_kbk - 0.002, 0.999), (k, stats[k])


def test_both_decoder_steps_against_the_oracle():
    from oracle import bolmo_ref
    m = _model(17)
    w, ref = _oracle_layer(m, m.dec, "dec")
    e, value = to_np(m.e), to_np(m.value)
    hd, x = bolmo_ref.norm_add(bolmo_ref.linear(e, w["w_in"]), value, ref.w["norm1"], 1e-6)
    _, xf = ref.step(hd, x, out_norm=w["final_norm"])
    want = {"logits": bolmo_ref.linear(xf, w["lm_head"], bf16_out=False), "C": ref.state[0]}
    snap = _snap(m.dec)
    got = {}
    for fused in (False, True):
        _restore(m.dec, snap)
        _run(m, "dec", fused)
        got[fused] = {"logits": m.logits.clone(), "C": m.dec.state[0][0].clone()}
    stats = {k: (_stats(got[False][k], want[k]), _stats(got[True][k], want[k])) for k in want}
    print(stats)
    for k, ((e_kbk, c_kbk), (e_f, c_f)) in stats.items():
        assert e_f <= max(1.5 * e_kbk, 0.01) and c_f >= min(c_kbk - 0.002, 0.999), (k, stats[k])


def _everything(m):
    return [m.e, m.patch, m.boundary_logit, m.logits, m.out, *m.enc.state, *m.enc.nm[1], *m.dec.state, *m.dec.nm[1]]


def test_one_launch_for_both_steps_equals_the_two_launches_bit_for_bit():
    """bp_loc_encdec_step (a byte that opens no patch: encoder then decoder in one persistent launch) gives
    the outputs and new states of bp_loc_enc_step followed by bp_loc_dec_step exactly, launch after launch."""
    m = _model(9)
    snap_e, snap_d = _snap(m.enc), _snap(m.dec)
    for byte in (97, 3, 500):
        _restore(m.enc, snap_e)
        _restore(m.dec, snap_d)
        m.byte.fill_(byte)
        m.enc_step(0)
        m.dec_step(0)
        torch.cuda.synchronize()
        want = [t.clone() for t in _everything(m)]
        _restore(m.enc, snap_e)
        _restore(m.dec, snap_d)
        m.logits.zero_()
        m.out.zero_()
        m.e.zero_()
        m.encdec_step(0)
        torch.cuda.synchronize()
        got = _everything(m)
        bad = [i for i, (a, b) in enumerate(zip(got, want)) if not torch.equal(a, b)]
        assert not bad, (byte, bad)


def test_one_launch_for_both_steps_with_a_byte_outside_the_vocabulary_runs_neither_layer():
    m = _model(13)
    snap_e, snap_d = _snap(m.enc), _snap(m.dec)
    m.logits.fill_(1.0)
    m.out.fill_(7)
    m.byte.fill_(512)
    m.encdec_step(0)
    torch.cuda.synchronize()
    assert torch.isnan(m.e.float()).all() and torch.isnan(m.patch.float()).all()
    assert torch.isnan(m.boundary_logit).all()
    assert all(torch.equal(a, b) for a, b in zip((*m.enc.state, *m.enc.nm[1]), snap_e))
    assert all(torch.equal(a, b) for a, b in zip((*m.dec.state, *m.dec.nm[1]), snap_d))
    assert bool((m.logits == 1.0).all()) and bool((m.out == 7).all())
