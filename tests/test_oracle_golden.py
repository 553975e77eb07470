"""The CPU oracle against the golden vectors produced by the reference's own code
(tests/golden/make_golden.py): int8 quantizer, dequantizer, the tests' fp32 matmul reference, the
Triton int8 GEMV and the fused mLSTM kernels (fp32, Triton interpreter), and the accept kernel."""

from pathlib import Path

import numpy as np
import pytest

from oracle import mlstm_ref, skinny_ref
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16

G = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


def test_round_bf16_matches_bit_rounding_rules():
    vals = np.array([1.0, 1.00390625, 1.005859375, 1.0078125 + 2**-9, -3.0e38, 1e-40, np.inf, -0.0], np.float32)
    r = round_bf16(vals)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even (1 + 2^-8 is halfway, mantissa even -> down)
    assert r[2] == np.float32(1.0078125)
    assert np.isinf(r[6]) and np.signbit(r[7])
    assert np.array_equal(bf16_bits_to_f32(f32_to_bf16_bits(vals)), r)
    assert np.isnan(round_bf16(np.array([np.nan], np.float32)))[0]


def test_int8_quantizer_is_bit_exact():
    w = bf16_bits_to_f32(G["q8_w"])
    q, s = skinny_ref.quantize_rowwise_int8(w)
    assert np.array_equal(q, G["q8_q"])
    assert np.array_equal(f32_to_bf16_bits(s), G["q8_scale"])
    assert np.array_equal(skinny_ref.dequantize("int8", q, s), G["q8_deq"])


@pytest.mark.parametrize("key", sorted(k[:-2] for k in G.files if k.startswith("lin_") and k.endswith("_y")))
def test_fp32_reference_matmul(key):
    kind = key.split("_")[1]
    x = bf16_bits_to_f32(G[key + "_x"])
    w = bf16_bits_to_f32(G[key + "_w"])
    wd = skinny_ref.dequantize("bf16", w) if kind == "bf16" else skinny_ref.dequantize(
        "int8", *skinny_ref.quantize_rowwise_int8(w))
    y = skinny_ref.linear_ref(x, wd, exact=True)
    assert skinny_ref.rel_normwise(y, G[key + "_y"]) < 1e-6


@pytest.mark.parametrize("r", [32, 16])
def test_int4_quantizer_packing_and_dequantizer_are_bit_exact(r):
    w = bf16_bits_to_f32(G["q4_w"])
    packed, scale, zero = skinny_ref.quantize_int4(w, tile_rows=r)
    assert np.array_equal(packed, G[f"q4_r{r}_packed"])
    assert np.array_equal(f32_to_bf16_bits(scale), G[f"q4_r{r}_scale"])
    assert np.array_equal(zero.view(np.uint16), G[f"q4_r{r}_zero"])
    assert np.array_equal(skinny_ref.unpack_int4(packed, w.shape[0]), G[f"q4_r{r}_codes"])
    assert np.array_equal(skinny_ref.pack_int4(G[f"q4_r{r}_codes"], r), packed)
    assert np.array_equal(skinny_ref.dequantize("int4", packed, scale, zero), G[f"q4_r{r}_deq"])


def test_int4_fp32_reference_matmul():
    w = bf16_bits_to_f32(G["q4_w"])
    wd = skinny_ref.dequantize("int4", *skinny_ref.quantize_int4(w))
    y = skinny_ref.linear_ref(bf16_bits_to_f32(G["q4lin_x"]), wd, exact=True)
    assert skinny_ref.rel_normwise(y, G["q4lin_y"]) < 1e-6


@pytest.mark.parametrize("key", sorted(k[:-2] for k in G.files if k.startswith("gemv_") and k.endswith("_y")))
def test_int8_gemv_golden(key):
    x = bf16_bits_to_f32(G[key + "_x"])
    y_ref = bf16_bits_to_f32(G[key + "_y"])
    y = skinny_ref.linear_ref(x, skinny_ref.dequantize("int8", G[key + "_q"], bf16_bits_to_f32(G[key + "_scale"])),
                              exact=True)
    assert skinny_ref.close_int8(y_ref, y)
    # The reference's bf16 output is the fp32 accumulator cast to bf16: within one bf16 step of the exact
    # value (the Triton CPU interpreter truncates that cast where the GPU rounds to nearest, so the
    # golden values may sit one step below the rounded exact value; one step <= 2^-7 |y|).
    step = np.abs(y) * 2.0**-7 + 1e-6
    assert (np.abs(y - y_ref) <= step).all()


MS_KEYS = sorted({k.rsplit("_", 1)[0] for k in G.files if k.startswith("ms_") and k.endswith("_h")})


@pytest.mark.parametrize("key", MS_KEYS)
def test_mlstm_fp32_matches_reference_kernels(key):
    q, k, v, i, f = (G[f"{key}_{n}"] for n in "qkvif")
    state = (G[key + "_c0"][0], G[key + "_n0"][0], G[key + "_m0"][0, :, 0])
    dq = q.shape[-1]
    h, ns, msv = mlstm_ref.multistep_fw(state, q, k, v, i[..., 0], f[..., 0], dq ** -0.5, 1e-6, bf16=False)
    assert skinny_ref.rel_normwise(h, G[key + "_h"]) < 5e-6  # the reference tests' fp32 bar
    assert np.array_equal(ns, G[key + "_nstart"]) and np.array_equal(msv, G[key + "_mstart"])
    for length in range(q.shape[0]):
        c, n, m = mlstm_ref.lazy_commit(state, k, v, i[..., 0], f[..., 0], length, bf16=False)
        assert skinny_ref.rel_normwise(c, G[f"{key}_L{length}_c"][0]) < 1e-6
        assert skinny_ref.rel_normwise(n, G[f"{key}_L{length}_n"][0]) < 1e-6
        assert skinny_ref.rel_normwise(m, G[f"{key}_L{length}_m"][0, :, 0]) < 1e-6


@pytest.mark.parametrize("j", range(4))
def test_accept_known_answers(j):
    out = mlstm_ref.accept(G["acc_ids"], G[f"acc_tok{j}"], 6, 6, 8)
    assert np.array_equal(out, G[f"acc_out{j}"])


def test_bf16_scan_rounds_where_the_reference_rounds():
    """Teeth for the bf16 precision model: dropping any one of the bf16 roundings moves h."""
    rng = np.random.default_rng(0)
    nh, dq, dv, t = 2, 64, 16, 6
    q, k = (round_bf16(rng.standard_normal((t, nh, dq)).astype(np.float32)) for _ in range(2))
    v = round_bf16(rng.standard_normal((t, nh, dv)).astype(np.float32))
    i, f = (rng.standard_normal((t, nh)).astype(np.float32) * 2 for _ in range(2))
    state = (np.zeros((nh, dq, dv), np.float32), np.zeros((nh, dq), np.float32), np.zeros(nh, np.float32))
    h_bf, st_bf, _ = mlstm_ref.scan(state, q, k, v, i, f, dq ** -0.5, 1e-6, bf16=True)
    h_32, st_32, _ = mlstm_ref.scan(state, q, k, v, i, f, dq ** -0.5, 1e-6, bf16=False)
    # bf16 rounding of the products is visible but small
    assert 1e-4 < skinny_ref.rel_normwise(st_bf[0], st_32[0]) < 2e-2
    assert np.array_equal(h_bf, round_bf16(h_bf))  # h is bf16-valued
