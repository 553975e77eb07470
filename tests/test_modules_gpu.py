"""GPU checks of the operator modules, following the reference's tests/test_quant_int8.py and
tests/test_skinny_integration.py: the int8 GEMV on real and odd shapes, Int8Linear for several row
counts with and without bias, empty inputs, CUDA-graph replay, the SkinnyLinear swap on a toy
OLMo-shaped model, fp32 activations taking the dequantized path."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from byteprof_b200.optim.skinny_linear import SkinnyLinear
from byteprof_b200.quant.int8 import gemv_int8, quantize_rowwise_int8
from byteprof_b200.quant.integrate import Int8Linear, apply_quantization
from helpers import to_np
from oracle import skinny_ref

pytestmark = pytest.mark.gpu


def _ref(x, q, s, bias=None):
    y = skinny_ref.linear_ref(to_np(x), skinny_ref.dequantize("int8", to_np(q), to_np(s)), exact=True)
    return y if bias is None else y + to_np(bias)


def _close(y, ref):
    assert y.dtype == torch.bfloat16
    assert skinny_ref.close_int8(to_np(y), ref)


@pytest.mark.parametrize("n,k", [(1024, 2048), (2048, 2048), (2816, 2048), (2048, 2816), (8192, 2048), (2048, 8192)])
def test_gemv_real_shapes_batch_one(n, k):
    q, s = quantize_rowwise_int8((torch.randn(n, k) * 0.02).to("cuda", torch.bfloat16))
    x = torch.randn(1, k, device="cuda", dtype=torch.bfloat16)
    _close(gemv_int8(x, q, s), _ref(x, q, s))


@pytest.mark.parametrize("n,k", [(2048, 2048), (4096, 2048), (2048, 8192), (4104, 2048), (8192, 2048)])
def test_gemv_is_skinny_mm_at_one_row_bit_for_bit(n, k, monkeypatch):
    """gemv_int8 is skinny_mm at M = 1: bit-identical to it on its default route and with the tensor-core
    kernel forced (BP_SKINNY_PATH=tc), since both int8 kernels it can take sum exactly."""
    from byteprof_b200.optim.skinny import skinny_mm

    g = torch.Generator().manual_seed(n + k)
    q, s = quantize_rowwise_int8((torch.randn(n, k, generator=g) * 0.02).to("cuda", torch.bfloat16))
    x = torch.randn(1, k, generator=g).to("cuda", torch.bfloat16)
    y = gemv_int8(x, q, s)
    _close(y, _ref(x, q, s))
    assert torch.equal(y, skinny_mm(x, q, s))
    monkeypatch.setenv("BP_SKINNY_PATH", "tc")
    want = skinny_mm(x, q, s)
    monkeypatch.delenv("BP_SKINNY_PATH", raising=False)
    assert torch.equal(y, want)


@pytest.mark.parametrize("n,k", [(37, 1000), (1, 8), (3, 129), (1025, 2049), (16, 2047), (7, 5000), (24, 128)])
def test_gemv_odd_sizes_not_multiples_of_block(n, k):
    q, s = quantize_rowwise_int8((torch.randn(n, k) * 0.05).to("cuda", torch.bfloat16))
    x = torch.randn(1, k, device="cuda", dtype=torch.bfloat16)
    _close(gemv_int8(x, q, s), _ref(x, q, s))
    for cfg in ((1, 256, 1), (8, 1024, 8)):  # cfg is accepted and ignored
        _close(gemv_int8(x, q, s, cfg), _ref(x, q, s))


@pytest.mark.parametrize("m", [1, 2, 5, 33, 300])
@pytest.mark.parametrize("n,k,bias", [(2048, 2048, True), (2816, 2048, False), (37, 1000, True)])
def test_int8linear_all_row_counts_vs_fp32_reference(m, n, k, bias):
    lin = nn.Linear(k, n, bias=bias, dtype=torch.bfloat16, device="cuda")
    mod = Int8Linear(lin)
    x = torch.randn(m, 1, k, device="cuda", dtype=torch.bfloat16)
    y = mod(x)
    assert y.shape == (m, 1, n)
    _close(y.reshape(m, n), _ref(x.reshape(m, k), mod.q, mod.scale, lin.bias if bias else None))


def test_int8linear_empty_input():
    mod = Int8Linear(nn.Linear(256, 64, bias=True, dtype=torch.bfloat16, device="cuda"))
    for shape in ((0, 256), (0, 1, 256)):
        y = mod(torch.empty(*shape, device="cuda", dtype=torch.bfloat16))
        assert y.shape == (*shape[:-1], 64) and y.numel() == 0


def test_gemv_inside_cuda_graph_matches_eager():
    q, s = quantize_rowwise_int8((torch.randn(2048, 2048) * 0.02).to("cuda", torch.bfloat16))
    x = torch.randn(1, 2048, device="cuda", dtype=torch.bfloat16)
    gemv_int8(x, q, s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = gemv_int8(x, q, s)
    x.copy_(torch.randn_like(x))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, gemv_int8(x, q, s))


class _Block(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.self_attn = nn.ModuleDict({n: nn.Linear(d, d, bias=False) for n in ("q_proj", "k_proj", "v_proj", "o_proj")})
        self.mlp = nn.ModuleDict({"gate_proj": nn.Linear(d, 2 * d, bias=False), "up_proj": nn.Linear(d, 2 * d, bias=False),
                                  "down_proj": nn.Linear(2 * d, d, bias=False)})


class _Toy(nn.Module):
    def __init__(self, d=256):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Block(d) for _ in range(2)])
        self.lm_head = nn.Linear(d, 64, bias=False)


def _toy(seed=0):
    torch.manual_seed(seed)
    return _Toy().to("cuda", torch.bfloat16)


@pytest.mark.parametrize("scheme", ["bf16_wo", "int8_wo"])
def test_apply_quantization_with_the_skinny_kernel_swaps_selected_linears(scheme):
    m = _toy()
    stats = apply_quantization(m, "blocks", scheme, 128, None, None, "skinny")
    assert stats["kernel"] == "skinny" and stats["n_linears"] == 14
    assert sum(isinstance(x, SkinnyLinear) for x in m.modules()) == 14 and isinstance(m.lm_head, nn.Linear)
    ref = _toy()
    for rows in (1, 5, 100):  # kernel, kernel, dequantized fallback
        xr = torch.randn(rows, 256, device="cuda", dtype=torch.bfloat16)
        a = m.model.layers[0].self_attn["q_proj"](xr).float()
        b = ref.model.layers[0].self_attn["q_proj"](xr).float()
        assert a.shape == b.shape == (rows, 256)
        tol = {"bf16_wo": 1e-2, "int8_wo": 0.1}[scheme]
        assert (a - b).abs().max() < tol * b.abs().max()
    assert m.model.layers[0].self_attn["q_proj"](torch.empty(0, 256, device="cuda", dtype=torch.bfloat16)).shape == (0, 256)
    assert m.model.layers[0].self_attn["q_proj"].weight.dtype == torch.bfloat16


def test_skinny_int8_uses_the_same_quantized_weights_as_the_default_int8():
    lin = nn.Linear(512, 128, bias=False, dtype=torch.bfloat16, device="cuda")
    a, b = Int8Linear(lin), SkinnyLinear(lin, "int8_wo")
    assert torch.equal(a.q, b.q) and torch.equal(a.scale, b.scale)
    x = torch.randn(1, 512, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(a(x), b(x))  # one kernel family: identical bits


def test_skinny_linear_inside_a_cuda_graph_with_bias():
    lin = nn.Linear(256, 96, bias=True, dtype=torch.bfloat16, device="cuda")
    for scheme in ("bf16_wo", "int8_wo"):
        m = SkinnyLinear(lin, scheme)
        x = torch.randn(3, 1, 256, device="cuda", dtype=torch.bfloat16)
        eager = m(x)
        with torch.inference_mode():
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                m(x)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                y = m(x)
            x.copy_(torch.randn_like(x))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(y, m(x))
        assert eager.shape == (3, 1, 96)


def test_fp32_activations_use_the_dequantized_weights():
    lin = nn.Linear(256, 64, bias=False, dtype=torch.float32, device="cuda")
    m = SkinnyLinear(lin, "int8_wo")
    x = torch.randn(3, 256, device="cuda", dtype=torch.float32)
    y = m(x)
    assert y.dtype == torch.float32
    assert torch.allclose(y, x @ m.dequantized(torch.float32).T, atol=1e-5, rtol=1e-5)
    assert (y - lin(x)).abs().max() < 0.1 * lin(x).abs().max()
    ref = skinny_ref.linear_ref(to_np(x), to_np(m.dequantized(torch.float32)), exact=True)
    assert np.abs(to_np(y) - ref).max() < 1e-4
