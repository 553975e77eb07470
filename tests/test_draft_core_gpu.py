"""The drafting helpers of byteprof_b200.optim.draft_core with the sm_100a step and the device commit.

Follows the reference's tests/test_draft_kernels_gpu.py: the scan with history, driven by the library step
(here mlstm_step_into on bp_mlstm_scan), fills every slot with the state of the sequential steps; the commit
selects the slot read on the device, also inside a CUDA graph whose slot changes between replays; the
accepted length on the device. Beyond that: the torch references of the fused pair (scan_without_history,
lazy_commit_state) with the device step give bit for bit what the fused kernels (multistep_fw,
lazy_commit) give, and the history slots agree with the CPU oracle."""

from functools import partial

import pytest
import torch

from byteprof_b200.optim import draft_core as core
from byteprof_b200.optim import draft_fused
from helpers import to_np
from oracle import mlstm_ref
from oracle.skinny_ref import rel_normwise

pytestmark = pytest.mark.gpu
STEP = partial(core.mlstm_step_into, eps=1e-6)


def _inputs(s, dtype, nh, dq, dv, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *shape, dt=dtype: torch.randn(*shape, generator=g, device="cuda", dtype=dt)  # noqa: E731
    return (r(s, nh, dq), r(s, nh, dq), r(s, nh, dv), r(s, nh, 1, dt=torch.float32) * 2,
            r(s, nh, 1, dt=torch.float32) * 2 + 1,
            (r(1, nh, dq, dv, dt=torch.float32) * 0.1, r(1, nh, dq, dt=torch.float32) * 0.1,
             r(1, nh, 1, dt=torch.float32)))


def _hist(slots, nh, dq, dv):
    return (torch.zeros(slots, 1, nh, dq, dv, device="cuda"), torch.zeros(slots, 1, nh, dq, device="cuda"),
            torch.zeros(slots, 1, nh, 1, device="cuda"))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("nh,dq,dv", [(16, 128, 128), (4, 512, 512)])
def test_scan_with_history_fills_the_slots_of_the_sequential_steps(dtype, nh, dq, dv):
    s = 5
    q, k, v, i, f, state = _inputs(s, dtype, nh, dq, dv)
    hist, hbuf = _hist(9, nh, dq, dv), torch.zeros(9, nh, dv, dtype=dtype, device="cuda")
    cur = tuple(t.clone() for t in state)
    core.scan_with_history(STEP, cur, hist, s, q, k, v, i, f, hbuf)
    assert all(torch.equal(a, b) for a, b in zip(cur, state))  # the scan leaves the current state alone
    prev = state
    for j in range(s):
        new = tuple(torch.empty_like(t) for t in state)
        h = torch.empty(1, nh, dv, dtype=dtype, device="cuda")
        core.mlstm_step_into(prev, new, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], h, eps=1e-6)
        assert torch.equal(h, hbuf[j:j + 1])
        assert all(torch.equal(a, t[j]) for a, t in zip(new, hist))
        prev = new
    # the history against the CPU oracle
    _, _, states = mlstm_ref.scan((to_np(state[0])[0], to_np(state[1])[0], to_np(state[2]).reshape(-1)), to_np(q),
                                  to_np(k), to_np(v), to_np(i)[..., 0], to_np(f)[..., 0], dq ** -0.5, 1e-6,
                                  dtype == torch.bfloat16, keep_states=True)
    for j in range(s):
        for a, b in zip(hist, states[j]):
            assert rel_normwise(to_np(a[j]).reshape(b.shape), b) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_torch_references_of_the_fused_pair_equal_the_fused_kernels(dtype):
    nh, dq, dv, s = 4, 512, 512, 7
    q, k, v, i, f, state = _inputs(s, dtype, nh, dq, dv, seed=4)
    hbuf = torch.zeros(8, nh, dv, dtype=dtype, device="cuda")
    start = core.scan_without_history(STEP, state, s, q, k, v, i, f, hbuf)
    assert all(torch.equal(a, b) for a, b in zip(start, state))
    fused_h = torch.zeros(8, nh, dv, dtype=dtype, device="cuda")
    ns, ms = torch.zeros(nh, dq, device="cuda"), torch.zeros(nh, device="cuda")
    cur = tuple(t.clone() for t in state)
    draft_fused.multistep_fw(cur, q, k, v, i, f, fused_h, ns, ms, eps=1e-6)
    assert torch.equal(hbuf, fused_h)
    for slot in (0, 3, s - 1):
        ref = tuple(t.clone() for t in state)
        core.lazy_commit_state(STEP, ref, start, torch.tensor(slot, device="cuda"), q, k, v, i, f)
        fused = tuple(t.clone() for t in state)
        draft_fused.lazy_commit(fused, k, v, i, f, torch.tensor(slot, device="cuda"), ns, ms)
        assert all(torch.equal(a, b) for a, b in zip(ref, fused)), slot


@pytest.mark.parametrize("length_dtype", [torch.int64, torch.int32])
def test_commit_reads_the_slot_on_the_device_inside_a_graph(length_dtype):
    nh, dq, dv = 16, 128, 128
    hist = (torch.randn(9, 1, nh, dq, dv, device="cuda"), torch.randn(9, 1, nh, dq, device="cuda"),
            torch.randn(9, 1, nh, 1, device="cuda"))
    cur = tuple(torch.zeros_like(h[0]) for h in hist)
    length = torch.zeros((), dtype=length_dtype, device="cuda")
    core.commit_state(hist, cur, length)  # warm-up outside the capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        core.commit_state(hist, cur, length)
    for slot in (0, 3, 6, 8, 1):
        length.fill_(slot)
        g.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(c, h[slot]) for c, h in zip(cur, hist)), slot
    length.fill_(9)  # outside the history: NaN, nothing read
    g.replay()
    torch.cuda.synchronize()
    assert all(torch.isnan(c).all() for c in cur)
    del g


def test_commit_of_unaligned_states_takes_the_element_path():
    nh, dq, dv = 3, 5, 7  # counts that are not multiples of four
    hist = (torch.randn(4, 1, nh, dq, dv, device="cuda"), torch.randn(4, 1, nh, dq, device="cuda"),
            torch.randn(4, 1, nh, 1, device="cuda"))
    cur = tuple(torch.zeros_like(h[0]) for h in hist)
    core.commit_state(hist, cur, torch.tensor([2], device="cuda"))
    torch.cuda.synchronize()
    assert all(torch.equal(c, h[2]) for c, h in zip(cur, hist))


def test_commit_rejects_bad_tensors():
    hist = tuple(torch.zeros(2, 1, 4, device="cuda") for _ in range(3))
    cur = tuple(torch.zeros(1, 4, device="cuda") for _ in range(3))
    with pytest.raises(ValueError):
        core.commit_state(hist, cur, torch.zeros((), dtype=torch.float32, device="cuda"))
    with pytest.raises(ValueError):
        core.commit_state(hist, tuple(torch.zeros(1, 5, device="cuda") for _ in range(3)),
                          torch.zeros((), dtype=torch.int64, device="cuda"))


def test_accepted_length_on_the_device():
    ids = torch.tensor([10, 5, 6, 7, 8, 9], device="cuda")
    assert int(core.accepted_length_t(ids, torch.tensor([5, 6, 99, 8, 9, 3], device="cuda"), 6)) == 2
    assert int(core.accepted_length_t(ids, torch.tensor([5, 6, 7, 8, 9 + 260, 3], device="cuda"), 6)) == 4
    assert int(core.accepted_length_t(ids, torch.tensor([5, 6, 7, 8, 9, 3], device="cuda"), 6)) == 5
