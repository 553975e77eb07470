"""GPU parity of the fused mLSTM recurrence (bp_mlstm_scan) against the CPU oracle.

Follows the reference's tests/test_fused_kernels_gpu.py (multistep outputs and lazy commit for
T in {1, 2, 5, 9, 17, 33} and every L, head dims 64 and 128, fp32 and bf16; the pass never writes the
state; a CUDA graph with a dynamic L; the accept kernel's known answers), plus the BASELINE cell:
4 heads, dk = dv = 512, T in {1, 8, 64, 256} from a zero state, state within 1e-3 relative.
Error measure: normwise max|a - b| / max|b| (the reference's `rel`)."""

import numpy as np
import pytest
import torch

from byteprof_b200.optim import draft_core, draft_fused
from helpers import bf16_step_close, to_np
from oracle import mlstm_ref
from oracle.skinny_ref import rel_normwise

pytestmark = pytest.mark.gpu

NH, DV = 16, 128


def rand_inputs(t, dtype, seed=0, nh=NH, dq=64, dv=DV, gate_dtype=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    gd = gate_dtype or dtype
    r = lambda *shape, dt=dtype: torch.randn(*shape, generator=g, device="cuda", dtype=dt)  # noqa: E731
    return (r(t, nh, dq), r(t, nh, dq), r(t, nh, dv), r(t, nh, 1, dt=gd) * 2, r(t, nh, 1, dt=gd) * 2,
            (r(1, nh, dq, dv, dt=torch.float32) * 0.1, r(1, nh, dq, dt=torch.float32) * 0.1,
             r(1, nh, 1, dt=torch.float32)))


def oracle_scan(state, q, k, v, i, f, bf16, n_steps=None, keep_states=False):
    st = (to_np(state[0])[0], to_np(state[1])[0], to_np(state[2]).reshape(-1))
    dq = q.shape[-1]
    return mlstm_ref.scan(st, to_np(q), to_np(k), to_np(v), to_np(i)[..., 0], to_np(f)[..., 0], dq ** -0.5, 1e-6,
                          bf16, n_steps=n_steps, keep_states=keep_states)


@pytest.mark.parametrize("dq", (64, 128))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_multistep_and_lazy_commit_for_every_t_and_l(dtype, dq):
    bf16 = dtype == torch.bfloat16
    for t in (1, 2, 5, 9, 17, 33):
        q, k, v, i, f, state = rand_inputs(t, dtype, seed=t, dq=dq)
        h_ref, _, states = oracle_scan(state, q, k, v, i, f, bf16, keep_states=True)
        cur = tuple(x.clone() for x in state)
        hbuf = torch.zeros(40, NH, DV, dtype=dtype, device="cuda")
        ns, ms = torch.zeros(NH, dq, device="cuda"), torch.zeros(NH, device="cuda")
        draft_fused.multistep_fw(cur, q, k, v, i, f, hbuf, ns, ms, eps=1e-6)
        assert all(torch.equal(a, b) for a, b in zip(cur, state))  # the pass never writes the state
        assert torch.equal(ns, state[1][0]) and torch.equal(ms, state[2].reshape(-1))
        assert (hbuf[t:] == 0).all()
        if bf16:
            ok, worst, exact = bf16_step_close(to_np(hbuf[:t]), h_ref)
            assert ok, (t, worst, exact)
        else:
            err = rel_normwise(to_np(hbuf[:t]), h_ref)
            assert err < 1e-5, (t, err)
        for length in range(t):
            cur2 = tuple(x.clone() for x in state)
            draft_fused.lazy_commit(cur2, k, v, i, f, torch.tensor(length, device="cuda"), ns, ms)
            for a, b in zip(cur2, states[length]):
                e = rel_normwise(to_np(a).reshape(b.shape), b)
                assert e < 1e-5, (t, length, e)


def test_fp32_outputs_agree_to_fp32_rounding():
    q, k, v, i, f, state = rand_inputs(9, torch.float32)
    h_ref, _, _ = oracle_scan(state, q, k, v, i, f, False)
    hbuf = torch.zeros(9, NH, DV, device="cuda")
    ns, ms = torch.zeros(NH, 64, device="cuda"), torch.zeros(NH, device="cuda")
    draft_fused.multistep_fw(state, q, k, v, i, f, hbuf, ns, ms, eps=1e-6)
    assert rel_normwise(to_np(hbuf), h_ref) < 5e-6


def test_lazy_commit_in_a_graph_with_a_dynamic_length_and_in_place_state():
    t = 7
    q, k, v, i, f, state = rand_inputs(t, torch.bfloat16, seed=3)
    _, _, states = oracle_scan(state, q, k, v, i, f, True, keep_states=True)
    cur = tuple(x.clone() for x in state)
    start = tuple(x.clone() for x in state)
    hbuf = torch.zeros(8, NH, DV, dtype=torch.bfloat16, device="cuda")
    ns, ms = torch.zeros(NH, 64, device="cuda"), torch.zeros(NH, device="cuda")
    length = torch.zeros((), dtype=torch.long, device="cuda")
    draft_fused.multistep_fw(cur, q, k, v, i, f, hbuf, ns, ms, eps=1e-6)
    draft_fused.lazy_commit(cur, k, v, i, f, length, ns, ms)
    for a, b in zip(cur, start):
        a.copy_(b)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        draft_fused.multistep_fw(cur, q, k, v, i, f, hbuf, ns, ms, eps=1e-6)
        draft_fused.lazy_commit(cur, k, v, i, f, length, ns, ms)
    for length_v in (0, 3, t - 1, 1):
        for a, b in zip(cur, start):
            a.copy_(b)
        length.fill_(length_v)
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(cur, states[length_v]):
            assert rel_normwise(to_np(a).reshape(b.shape), b) < 1e-5, length_v


def test_length_beyond_t_is_clamped():
    t = 4
    q, k, v, i, f, state = rand_inputs(t, torch.float32, seed=11)
    _, last, _ = oracle_scan(state, q, k, v, i, f, False)
    cur = tuple(x.clone() for x in state)
    ns, ms = state[1][0].clone(), state[2].reshape(-1).clone()
    draft_fused.lazy_commit(cur, k, v, i, f, torch.tensor(50, device="cuda"), ns, ms)
    for a, b in zip(cur, last):
        assert rel_normwise(to_np(a).reshape(b.shape), b) < 1e-5


@pytest.mark.parametrize("t", [1, 8, 64, 256])
def test_baseline_cell_4_heads_512_from_zero_state(t):
    """NH=4, dk=dv=512, q,k,v ~ N(0,1)/sqrt(512) bf16, i ~ N(0,1), f ~ N(0,1) + 3 fp32."""
    nh, d = 4, 512
    g = torch.Generator(device="cuda").manual_seed(1000 + t)
    r = lambda *s: torch.randn(*s, generator=g, device="cuda")  # noqa: E731
    q, k, v = ((r(t, nh, d) / d ** 0.5).to(torch.bfloat16) for _ in range(3))
    i, f = r(t, nh, 1), r(t, nh, 1) + 3.0
    state = (torch.zeros(1, nh, d, d, device="cuda"), torch.zeros(1, nh, d, device="cuda"),
             torch.zeros(1, nh, 1, device="cuda"))
    out = tuple(torch.empty_like(x) for x in state)
    h = torch.empty(t, nh, d, dtype=torch.bfloat16, device="cuda")
    draft_core.mlstm_scan(state, q, k, v, i, f, h, out, eps=1e-6)
    h_ref, last, _ = oracle_scan(state, q, k, v, i, f, True)
    for a, b in zip(out, last):
        assert rel_normwise(to_np(a).reshape(b.shape), b) < 1e-3  # the BASELINE bar, on the fp32 state
    ok, worst, exact = bf16_step_close(to_np(h), h_ref)
    assert ok, (worst, exact)


def test_step_into_equals_one_position_of_the_scan():
    q, k, v, i, f, state = rand_inputs(3, torch.bfloat16, seed=5, dq=128)
    prev = state
    for j in range(3):
        new = tuple(torch.empty_like(x) for x in state)
        h = torch.empty(1, NH, DV, dtype=torch.bfloat16, device="cuda")
        draft_core.mlstm_step_into(prev, new, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], h, eps=1e-6)
        h_ref, last, _ = oracle_scan(prev, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], True)
        assert bf16_step_close(to_np(h), h_ref)[0]
        for a, b in zip(new, last):
            assert rel_normwise(to_np(a).reshape(b.shape), b) < 1e-5
        prev = new


def test_head_dims_256_and_fp32_gates_with_bf16_inputs():
    q, k, v, i, f, state = rand_inputs(6, torch.bfloat16, seed=8, nh=3, dq=256, dv=32, gate_dtype=torch.float32)
    h_ref, last, _ = oracle_scan(state, q, k, v, i, f, True)
    out = tuple(torch.empty_like(x) for x in state)
    h = torch.empty(6, 3, 32, dtype=torch.bfloat16, device="cuda")
    draft_core.mlstm_scan(state, q, k, v, i, f, h, out, eps=1e-6)
    assert bf16_step_close(to_np(h), h_ref)[0]
    for a, b in zip(out, last):
        assert rel_normwise(to_np(a).reshape(b.shape), b) < 1e-5


def test_accept_kernel_known_answers():
    ids = torch.tensor([10, 5, 6, 7, 8, 9], device="cuda")
    for tokl, want in (([5, 6, 99, 8, 9, 3], 2), ([5, 6, 7, 8, 9 + 260, 3], 4), ([1, 6, 7, 8, 9, 3], 0),
                       ([5, 6, 7, 8, 9, 3], 5)):
        tok = torch.tensor(tokl, device="cuda")
        out = torch.zeros(8, dtype=torch.long, device="cuda")
        draft_fused.accept(ids, tok, out, 6, 6)
        assert int(out[6]) == want
        assert out[:6].tolist() == tokl
        assert np.array_equal(out.cpu().numpy(), mlstm_ref.accept(ids.cpu().numpy(), tokl, 6, 6, 8))
