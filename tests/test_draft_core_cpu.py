"""Exactness of the drafting round logic in byteprof_b200.optim.draft_core on a small CPU model.

The properties are those of the reference's toy-model test (byteprof tests/test_draft_toy.py): a tiny
random byte model with fused (byte, boundary flag) ids, a stateful subword automaton, a recurrent encoder
and decoder layer and a recurrent "global" update on flagged positions, decoded one id at a time ("plain")
and by `rounds_loop` with random, all-wrong and all-right drafts; both the history form (scan_with_history
+ commit_state) and the lazy form (scan_without_history + lazy_commit_state) of the round must give the
plain bytes exactly. The model, automaton and drafters here are this repository's own; only the drafting
functions under test come from the package. CPU only, fp32.
"""

from __future__ import annotations

import random

import pytest
import torch
import torch.nn as nn

from byteprof_b200.optim import draft_core as core

OFF, FLAG = 4, 260  # byte id = byte + OFF; a boundary-flagged id adds FLAG
NBYTES = 8
NSUB = 5
D, NH, DQ, DV = 16, 2, 4, 8
VOCAB = 2 * FLAG
EOS = 2
EOS_IDS = (EOS, EOS + FLAG)
NO_BPE_END = -1


def cell(prev, new, q, k, v, i, f, h):
    """A small matrix-memory recurrence; writes `new` and `h`, leaves `prev` alone."""
    c0, n0, m0 = prev
    a, b = torch.sigmoid(f), torch.sigmoid(i)  # (1, NH, 1)
    new[0].copy_(a[..., None] * c0 + b[..., None] * (k[..., :, None] * v[..., None, :]))
    new[1].copy_(a * n0 + b * k)
    new[2].copy_(a * m0 + b)
    num = torch.einsum("bhq,bhqv->bhv", q, new[0])
    den = (q * new[1]).sum(-1, keepdim=True).abs().clamp(min=1.0) + new[2].abs()
    h.copy_(num / den)


def zeros_state():
    return torch.zeros(1, NH, DQ, DV), torch.zeros(1, NH, DQ), torch.zeros(1, NH, 1)


def zeros_hist(slots):
    return torch.zeros(slots, 1, NH, DQ, DV), torch.zeros(slots, 1, NH, DQ), torch.zeros(slots, 1, NH, 1)


class Layer(nn.Module):
    def __init__(self):
        super().__init__()
        self.norm = nn.LayerNorm(D, elementwise_affine=False)
        self.proj = nn.Linear(D, 2 * NH * DQ + NH * DV + 2 * NH)  # q | k | v | i | f
        self.out = nn.Linear(NH * DV, D)
        self.ff = nn.Sequential(nn.Linear(D, 3 * D), nn.Tanh(), nn.Linear(3 * D, D))
        with torch.no_grad():  # a long memory with a strong read-out: a wrong state changes the bytes
            self.proj.weight.mul_(2.5)
            self.proj.bias[-NH:].fill_(2.0)
            self.out.weight.mul_(4.0)

    def project(self, x, s):
        p = self.proj(self.norm(x)).view(s, -1)
        a, b, c = NH * DQ, 2 * NH * DQ, 2 * NH * DQ + NH * DV
        return (p[:, :a].reshape(s, NH, DQ), p[:, a:b].reshape(s, NH, DQ), p[:, b:c].reshape(s, NH, DV),
                p[:, c:c + NH].reshape(s, NH, 1), p[:, c + NH:].reshape(s, NH, 1))

    def finish(self, x, hs, s):
        x = x + self.out(hs[:s].reshape(1, s, NH * DV))
        return x + self.ff(x)

    def one(self, x, state):
        """One position; the state advances in place."""
        q, k, v, i, f = self.project(x, 1)
        nxt = tuple(torch.empty_like(t) for t in state)
        h = torch.empty(1, NH, DV)
        cell(state, nxt, q, k, v, i, f, h)
        for dst, src in zip(state, nxt):
            dst.copy_(src)
        return self.finish(x, h, 1)

    def round(self, x, s, state, hist, hbuf, lazy):
        """S positions; history form writes the slots, lazy form returns what lazy_commit_state needs."""
        q, k, v, i, f = self.project(x, s)
        saved = None
        if lazy:
            saved = (core.scan_without_history(cell, state, s, q, k, v, i, f, hbuf), q, k, v, i, f)
        else:
            core.scan_with_history(cell, state, hist, s, q, k, v, i, f, hbuf)
        return self.finish(x, hbuf, s), saved


class Model(nn.Module):
    def __init__(self, seed):
        super().__init__()
        torch.manual_seed(seed)
        self.emb = nn.Embedding(VOCAB, D)
        self.sub = nn.Embedding(NSUB, D)
        self.enc, self.dec = Layer(), Layer()
        self.patch = nn.Linear(D, D)
        self.glob = nn.Linear(2 * D, D)
        self.inp = nn.Linear(D, D)
        self.norm = nn.LayerNorm(D)
        self.head = nn.Linear(D, VOCAB)
        with torch.no_grad():
            keep = torch.full((VOCAB,), -1e4)
            for b in range(NBYTES):
                keep[b + OFF] = keep[b + OFF + FLAG] = 0.0
            self.head.bias.copy_(keep)
            self.head.weight.mul_(4.0)
        self.eval()
        self.reset()

    def reset(self):
        self.es, self.ds = zeros_state(), zeros_state()
        self.g = torch.zeros(1, D)
        self.value = torch.zeros(1, 1, D)

    def open_patch(self, e0):
        self.g = torch.tanh(self.glob(torch.cat([self.g, self.patch(e0).reshape(1, D)], -1)))
        self.value = self.g.view(1, 1, D).clone()

    @torch.no_grad()
    def plain(self, byte_id, sub_id, boundary):
        x = self.emb(torch.tensor([[byte_id]])) + self.sub(torch.tensor([[sub_id]]))
        e = self.enc.one(x, self.es)
        if boundary:
            self.open_patch(e)
        y = self.dec.one(self.inp(e) + self.value, self.ds)
        return int(self.head(self.norm(y)).argmax(-1)[0, -1])


class Subwords:
    """A stateful subword id: depends on the previous byte, so a wrong rollback changes the outputs."""

    def step(self, state, byte):
        byte = byte - FLAG if byte >= FLAG else byte
        return byte, (5 * byte + 2 * state + 1) % NSUB


class Engine:
    def __init__(self, model, ks, lazy):
        self.m, self.k_values, self.lazy = model, tuple(ks), lazy
        slots = max(ks) + 1
        self.eh, self.dh = zeros_hist(slots), zeros_hist(slots)
        self.eb, self.db = torch.zeros(slots, NH, DV), torch.zeros(slots, NH, DV)

    @torch.no_grad()
    def run_round(self, k, boundary, ids, subs):
        m, s = self.m, k + 1
        ids_t = torch.tensor(ids)
        x = m.emb(ids_t.view(1, s)) + m.sub(torch.tensor(subs).view(1, s))
        e, esaved = m.enc.round(x, s, m.es, self.eh, self.eb, self.lazy)
        if boundary:
            m.open_patch(e[:, :1])
        y, dsaved = m.dec.round(m.inp(e) + m.value, s, m.ds, self.dh, self.db, self.lazy)
        tok = m.head(m.norm(y)).argmax(-1)[0]
        length = core.accepted_length_t(ids_t, tok, s)
        if self.lazy:
            core.lazy_commit_state(cell, m.es, esaved[0], length, *esaved[1:])
            core.lazy_commit_state(cell, m.ds, dsaved[0], length, *dsaved[1:])
        else:
            core.commit_state(self.eh, m.es, length)
            core.commit_state(self.dh, m.ds, length)
        return tok.tolist(), int(length)


def plain_ids(model, raw0, n_new, eos_ids=EOS_IDS):
    model.reset()
    aut = Subwords()
    st, sb = aut.step(0, raw0)
    raw, out = raw0, []
    for _ in range(n_new):
        flagged = raw >= FLAG
        raw = model.plain(raw - FLAG if flagged else raw, sb, flagged)
        out.append(raw)
        if raw in eos_ids:
            break
        st, sb = aut.step(st, raw)
    return out


def unflag(r):
    return r - FLAG if r >= FLAG else r


class Drafter:
    """Proposes from fn(k); `push` sees the atoms emitted each round."""

    def __init__(self, fn, on_push=None):
        self.fn, self.on_push = fn, on_push

    def reset(self, ctx, truth=None):
        pass

    def propose(self, k):
        return self.fn(k)

    def push(self, atoms):
        if self.on_push is not None:
            self.on_push(atoms)


def follower(truth, width=None):
    """A drafter that proposes the true continuation (width ids beyond the emitted position)."""
    pos = {"i": 0}

    def fn(k):
        return [core.atom_of(r, OFF, FLAG) for r in truth[pos["i"]:pos["i"] + (width or k)]]

    return Drafter(fn, lambda atoms: pos.__setitem__("i", pos["i"] + len(atoms))), pos


def drafted_ids(model, raw0, n_new, drafter, lazy, ks=(0, 1, 2, 3, 5, 8), k_max=8, eos_ids=EOS_IDS, stats=None,
                rounds=None):
    model.reset()
    aut = Subwords()
    st, sb = aut.step(0, raw0)
    tokens = [0] * (n_new + 3)
    drafter.reset([core.atom_of(raw0, OFF, FLAG)])
    n = core.rounds_loop(Engine(model, ks, lazy), aut, drafter, state=st, sub=sb, raw=raw0, tokens=tokens, n_tok=1,
                         stop_len=1 + n_new, eos_ids=eos_ids, bpe_end=NO_BPE_END, byte_offset=OFF,
                         boundary_offset=FLAG, k_max=k_max, stats=stats,
                         on_round=None if rounds is None else rounds.append)
    return tokens[1:n]


MODELS = [Model(seed) for seed in (0, 1, 2)]
RAW0 = (OFF + 3, OFF + 5 + FLAG)  # the first byte unflagged and flagged


@pytest.fixture(params=[False, True], ids=["history", "lazy"])
def lazy(request):
    return request.param


@pytest.mark.parametrize("n_new", [1, 2, 7, 40, 64])
def test_rounds_without_drafts_equal_plain_decoding(lazy, n_new):
    for m in MODELS:
        for r0 in RAW0:
            want = [unflag(r) for r in plain_ids(m, r0, n_new)]
            assert drafted_ids(m, r0, n_new, Drafter(lambda k: []), lazy, ks=(0,)) == want


def test_random_drafts_give_the_plain_bytes(lazy):
    rng = random.Random(11)
    for m in MODELS:
        for r0 in RAW0:
            want = [unflag(r) for r in plain_ids(m, r0, 80)]
            for _ in range(5):
                def fn(k):
                    return [rng.randrange(NBYTES) | (rng.randint(0, 1) << 8) for _ in range(rng.randint(0, k))]

                st = core.Stats()
                assert drafted_ids(m, r0, 80, Drafter(fn), lazy, stats=st) == want
                assert st.emitted == 80


def test_wrong_drafts_accept_nothing(lazy):
    for m in MODELS:
        for r0 in RAW0:
            truth = plain_ids(m, r0, 60)
            pos = {"i": 0}

            def fn(k):
                i = pos["i"]
                return [(unflag(truth[i + j]) - OFF + 1) % NBYTES for j in range(min(k, len(truth) - i - 1))]

            st = core.Stats()
            got = drafted_ids(m, r0, 60, Drafter(fn, lambda a: pos.__setitem__("i", pos["i"] + len(a))), lazy,
                              stats=st)
            assert got == [unflag(r) for r in truth]
            assert set(st.l_hist) == {0} and st.rounds == 60


def test_right_drafts_are_accepted_up_to_the_first_flagged_prediction(lazy):
    ended_at_flag = 0
    for m in MODELS:
        for r0 in RAW0:
            truth = plain_ids(m, r0, 90)
            d, _ = follower(truth)
            rounds, st = [], core.Stats()
            assert drafted_ids(m, r0, 90, d, lazy, stats=st, rounds=rounds) == [unflag(r) for r in truth]
            assert max(st.l_hist) > 0 and st.rounds < 90
            # a flagged prediction ends its round: nothing is emitted after it in the same round
            assert not [r for r in rounds if r["k"] and any(x >= FLAG for x in r["emitted"][:-1])]
            ended_at_flag += sum(1 for r in rounds if r["k"] and r["L"] < r["k"] and r["emitted"][-1] >= FLAG)
    assert ended_at_flag > 0


def test_the_length_cap_cuts_a_round_short(lazy):
    m, r0 = MODELS[0], RAW0[0]
    truth = plain_ids(m, r0, 50)
    for n_new in range(1, 30):
        d, _ = follower(truth)
        assert drafted_ids(m, r0, n_new, d, lazy) == [unflag(r) for r in truth[:n_new]]


def test_an_eos_inside_a_round_stops_decoding(lazy):
    m, r0 = MODELS[1], RAW0[0]
    truth = plain_ids(m, r0, 60)
    eos = (truth[17],)
    want = [unflag(r) for r in plain_ids(m, r0, 60, eos)]
    assert len(want) == truth.index(eos[0]) + 1
    d, _ = follower(truth)
    assert drafted_ids(m, r0, 60, d, lazy, eos_ids=eos) == want


def test_draft_lengths_without_a_graph_round_down(lazy):
    m, r0 = MODELS[2], RAW0[1]
    truth = plain_ids(m, r0, 70)
    d, _ = follower(truth, width=8)
    st = core.Stats()
    assert drafted_ids(m, r0, 70, d, lazy, ks=(0, 3), stats=st) == [unflag(r) for r in truth]
    assert set(st.by_k) <= {0, 3}


def _inputs(seed, s):
    g = torch.Generator().manual_seed(seed)
    r = lambda *shape: torch.randn(*shape, generator=g)  # noqa: E731
    return r(s, NH, DQ), r(s, NH, DQ), r(s, NH, DV), r(s, NH, 1), r(s, NH, 1), (r(1, NH, DQ, DV), r(1, NH, DQ),
                                                                              r(1, NH, 1))


def test_scan_with_history_is_the_sequential_steps_and_commit_takes_the_slot():
    s = 6
    q, k, v, i, f, cur = _inputs(3, s)
    before = tuple(t.clone() for t in cur)
    hist, hbuf = zeros_hist(8), torch.zeros(8, NH, DV)
    core.scan_with_history(cell, cur, hist, s, q, k, v, i, f, hbuf)
    assert all(torch.equal(a, b) for a, b in zip(cur, before))  # the current state waits for the commit
    prev = before
    for j in range(s):
        new, h = zeros_state(), torch.empty(1, NH, DV)
        cell(prev, new, q[j:j + 1], k[j:j + 1], v[j:j + 1], i[j:j + 1], f[j:j + 1], h)
        assert torch.equal(h, hbuf[j:j + 1])
        assert all(torch.equal(a, t[j]) for a, t in zip(new, hist))
        prev = new
    for slot in (0, 3, 5):
        core.commit_state(hist, cur, torch.tensor(slot))
        assert all(torch.equal(c, t[slot]) for c, t in zip(cur, hist))


def test_lazy_commit_rebuilds_each_history_slot_and_catches_the_usual_mistakes():
    s = 7
    q, k, v, i, f, cur = _inputs(5, s)
    hist, hbuf = zeros_hist(8), torch.zeros(8, NH, DV)
    core.scan_with_history(cell, cur, hist, s, q, k, v, i, f, hbuf)
    cur2, hbuf2 = tuple(t.clone() for t in cur), torch.zeros(8, NH, DV)
    start = core.scan_without_history(cell, cur2, s, q, k, v, i, f, hbuf2)
    assert torch.equal(hbuf, hbuf2) and all(torch.equal(a, b) for a, b in zip(cur, cur2))
    for slot in range(s):
        out = tuple(t.clone() for t in cur)
        core.lazy_commit_state(cell, out, start, torch.tensor(slot), q, k, v, i, f)
        assert all(torch.equal(a, t[slot]) for a, t in zip(out, hist)), slot
    good = tuple(t.clone() for t in cur)
    core.lazy_commit_state(cell, good, start, torch.tensor(2), q, k, v, i, f)
    for wrong in (1, 3):  # one position short, one too many
        bad = tuple(t.clone() for t in cur)
        core.lazy_commit_state(cell, bad, start, torch.tensor(wrong), q, k, v, i, f)
        assert not all(torch.equal(a, b) for a, b in zip(bad, good))
    bad = tuple(t.clone() for t in cur)  # recomputed from the advanced state instead of the start state
    core.lazy_commit_state(cell, bad, tuple(t[s - 1] for t in hist), torch.tensor(2), q, k, v, i, f)
    assert not all(torch.equal(a, b) for a, b in zip(bad, good))


def test_accepted_length_on_the_host_and_as_a_tensor_agree():
    rng = random.Random(1)
    for _ in range(300):
        k = rng.randint(0, 8)
        ids = [rng.randrange(4, 12) for _ in range(k + 1)]
        toks = [ids[j + 1] if rng.random() < 0.7 else rng.choice([rng.randrange(4, 12), rng.randrange(264, 272)])
                for j in range(k)] + [rng.randrange(4, 12)]
        host = core.accepted_length(ids, toks, k)
        dev = int(core.accepted_length_t(torch.tensor(ids), torch.tensor(toks), k + 1)) if k else 0
        assert host == dev
    ids = torch.tensor([10, 5, 6, 7, 8, 9])
    assert int(core.accepted_length_t(ids, torch.tensor([5, 6, 99, 8, 9, 3]), 6)) == 2
    assert int(core.accepted_length_t(ids, torch.tensor([5, 6, 7, 8, 9 + 260, 3]), 6)) == 4


def test_choose_k_and_atom_of():
    ks = (0, 1, 2, 4, 6, 8)
    assert [core.choose_k(n, ks, c) for n, c in ((0, 8), (3, 8), (8, 8), (8, 4), (7, 8))] == [0, 2, 8, 4, 6]
    assert core.atom_of(OFF + 7, OFF, FLAG) == 7
    assert core.atom_of(OFF + 7 + FLAG, OFF, FLAG) == 7 | 256
    assert core.atom_of(OFF - 1, OFF, FLAG) is None and core.atom_of(OFF + 256, OFF, FLAG) is None


def test_the_loop_rejects_a_device_length_that_disagrees():
    class Liar:
        k_values = (0, 2)

        def run_round(self, k, boundary, ids, subs):
            return [ids[1] if k else 5, 7, 9][:k + 1], 0  # confirms the first draft, reports L = 0

    with pytest.raises(RuntimeError, match="disagree"):
        core.rounds_loop(Liar(), Subwords(), Drafter(lambda k: [1, 2]), state=0, sub=0, raw=OFF, tokens=[0] * 10,
                         n_tok=1, stop_len=8, eos_ids=EOS_IDS, bpe_end=NO_BPE_END, byte_offset=OFF,
                         boundary_offset=FLAG, k_max=2)
