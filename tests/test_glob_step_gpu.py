"""The global-model step as one persistent kernel (bp_glob_step, csrc/glob_step.cu) against the same step
kernel by kernel (skinny GEMMs + bp_decode_attention + bp_rmsnorm_ex + bp_swiglu), from the same weights,
caches and position. The two differ only in the summation order of the matrix-vector products (CUDA-core
dot products here, tensor-core tiles there), so a bf16 rounding lands one step apart now and then; with
one block most outputs are bit-equal and all are within about one bf16 step, with the full 16 blocks the outputs stay within a few bf16
steps (normwise). Also: the position advances, the cache row of the position is written, a position
outside the cache writes NaN and nothing else, and repeated launches (and graph replays) agree."""

import numpy as np
import pytest
import torch

from byteprof_b200.optim.bolmo_e2e import EPS, BolmoDecoder
from byteprof_b200.optim.bolmo_local import rmsnorm
from byteprof_b200.optim.decode_ops import GlobStep
from helpers import to_np
from oracle import bolmo_ref

pytestmark = pytest.mark.gpu


def _setup(layers, pos, seed=5):
    m = BolmoDecoder(seed=seed, global_layers=layers)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    m.patch.copy_(torch.randn(1, m.d, generator=g, device="cuda").to(torch.bfloat16))
    for b in m.blocks:  # a cache already holding `pos` positions
        b.attn.k_cache.copy_(torch.randn(b.attn.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
        b.attn.v_cache.copy_(torch.randn(b.attn.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    caches = [(b.attn.k_cache.clone(), b.attn.v_cache.clone()) for b in m.blocks]
    m.pos.fill_(pos)
    return m, caches


def _kernels_path(m, pos):
    m.pos.fill_(pos)
    x = m.patch
    for b in m.blocks:
        x = b.step(x, m.pos, m.cos, m.sin)
    return rmsnorm(x, m.dec_in_norm, EPS)


def _restore(m, caches):
    for b, (k, v) in zip(m.blocks, caches):
        b.attn.k_cache.copy_(k)
        b.attn.v_cache.copy_(v)


def _compare(a, b):
    a, b = to_np(a), to_np(b)
    return float(np.abs(a - b).max() / np.abs(b).max()), float(np.mean(a == b))


@pytest.mark.parametrize("pos", [0, 200, 1023])
def test_one_block_matches_the_kernel_by_kernel_step(pos):
    m, caches = _setup(1, pos)
    ref = _kernels_path(m, pos)
    kc_ref = [b.attn.k_cache[pos].clone() for b in m.blocks]
    _restore(m, caches)
    m.pos.fill_(pos)
    m.glob_kernel(m.patch, m.value, m.pos)
    assert int(m.pos) == pos + 1
    err, exact = _compare(m.value, ref)
    assert err <= 2.0**-6 and exact >= 0.75, (err, exact)  # the final norms spread single-step flips
    for b, k in zip(m.blocks, kc_ref):
        e2, x2 = _compare(b.attn.k_cache[pos], k)
        assert e2 <= 2.0**-6 and x2 >= 0.95, (e2, x2)
        assert torch.equal(b.attn.k_cache[pos + 1:], caches[0][0][pos + 1:])  # nothing past p written


def test_sixteen_blocks_match_the_kernel_by_kernel_step():
    m, caches = _setup(16, 300)
    ref = _kernels_path(m, 300)
    _restore(m, caches)
    m.pos.fill_(300)
    m.glob_kernel(m.patch, m.value, m.pos)
    err, exact = _compare(m.value, ref)
    corr = float(np.corrcoef(to_np(m.value)[0], to_np(ref)[0])[0, 1])
    print({"err": err, "exact": exact, "corr": corr})
    assert corr >= 0.99 and err <= 0.1, (err, exact, corr)


def test_repeated_launches_and_graph_replays_agree():
    m, caches = _setup(2, 64)
    m.glob_kernel(m.patch, m.value, m.pos)
    first = m.value.clone()
    for _ in range(3):
        _restore(m, caches)
        m.pos.fill_(64)
        m.glob_kernel(m.patch, m.value, m.pos)
        assert torch.equal(m.value, first)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        m.glob_kernel(m.patch, m.value, m.pos)
    _restore(m, caches)
    m.pos.fill_(64)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(m.value, first) and int(m.pos) == 65


def test_a_position_outside_the_cache_writes_nan_and_nothing_else():
    m, caches = _setup(1, 0)
    m.pos.fill_(m.max_patches)
    m.glob_kernel(m.patch, m.value, m.pos)
    assert torch.isnan(m.value.float()).all() and int(m.pos) == m.max_patches
    assert torch.equal(m.blocks[0].attn.k_cache, caches[0][0]) and torch.equal(m.blocks[0].attn.v_cache, caches[0][1])


def test_each_block_of_the_persistent_kernel_against_the_oracle():
    """Block by block on the default (persistent) path: block i alone in the kernel, fed the oracle's input of
    block i, against the oracle's output of that block (both through the final RMSNorm the kernel applies),
    with the same caches holding 300 earlier positions. Every block within one bf16 step normwise and most
    outputs bit-equal: a per-block check that the statistical bar of the whole model cannot give."""
    pos = 300
    m, caches = _setup(16, pos, seed=9)
    w = {k: to_np(v) for k, v in m.weights().items()}
    ref = bolmo_ref.BolmoRef(w)
    for i, b in enumerate(m.blocks):
        ref.attn[i].k[:] = to_np(b.attn.k_cache)
        ref.attn[i].v[:] = to_np(b.attn.v_cache)
    ref.pos = pos
    x = to_np(m.patch)
    errs = []
    for i, b in enumerate(m.blocks):
        one = GlobStep([b], m.dec_in_norm, m.cos, m.sin, m.max_patches, EPS)
        xin = torch.from_numpy(x).to(device="cuda", dtype=torch.bfloat16)
        assert np.array_equal(to_np(xin), x)  # the oracle's bf16 activations go in exactly
        m.pos.fill_(pos)
        one(xin, m.value, m.pos)
        g = f"glob{i}."
        att = ref.attn[i](bolmo_ref.linear(x, w[g + "w_qkv"]), w[g + "q_norm"], w[g + "k_norm"], ref.cos, ref.sin, pos,
                          EPS)
        h = bolmo_ref.add_norm(bolmo_ref.linear(att, w[g + "w_o"]), x, w[g + "attn_norm"], EPS)
        dn = bolmo_ref.linear(bolmo_ref.swiglu(bolmo_ref.linear(h, w[g + "w_gu"])), w[g + "w_down"])
        x = bolmo_ref.add_norm(dn, h, w[g + "mlp_norm"], EPS)
        want = bolmo_ref.rmsnorm(x, w["dec_in_norm"], EPS)
        err, exact = _compare(m.value, torch.from_numpy(want))
        errs.append((i, round(err, 5), round(exact, 3)))
        assert err <= 2.0**-6 and exact >= 0.75, errs
    print(errs)
