"""Host-side logic of the operator API, on the CPU: argument validation (same errors as the
reference), the int8 and int4 weight preparation against the oracle (and the reference's own format
tests, tests/test_skinny.py:46-68), the module selection rules, the module swap, and that CPU tensors
are refused (there is no CPU path)."""

import numpy as np
import pytest
import torch
import torch.nn as nn

from byteprof_b200.optim import draft_fused, skinny
from byteprof_b200.optim.skinny_linear import SkinnyLinear
from byteprof_b200.quant import select
from byteprof_b200.quant.int8 import gemv_int8, quantize_rowwise_int8
from byteprof_b200.quant.integrate import Int8Linear, apply_quantization
from helpers import to_np
from oracle import skinny_ref


def test_quantizer_matches_oracle_bit_for_bit():
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(64, 512, generator=g) * 0.02).to(torch.bfloat16)
    w[5] = 0
    q, s = quantize_rowwise_int8(w)
    qo, so = skinny_ref.quantize_rowwise_int8(to_np(w))
    assert q.dtype == torch.int8 and s.dtype == torch.bfloat16
    assert np.array_equal(q.numpy(), qo) and np.array_equal(to_np(s), so)


@pytest.mark.parametrize("r", [32, 16])
def test_int4_preparation_matches_oracle_bit_for_bit(r):
    g = torch.Generator().manual_seed(11)
    w = (torch.randn(70, 384, generator=g) * 0.03).to(torch.bfloat16)
    w[3] = 0
    packed, scale, zero = skinny.quantize_int4(w, tile_rows=r)
    po, so, zo = skinny_ref.quantize_int4(to_np(w), tile_rows=r)
    assert packed.dtype == torch.uint8 and scale.dtype == torch.bfloat16 and zero.dtype == torch.float16
    assert np.array_equal(packed.numpy(), po) and np.array_equal(to_np(scale), so)
    assert np.array_equal(zero.numpy(), zo)
    assert np.array_equal(skinny.unpack_int4(packed, 70).numpy(), skinny_ref.unpack_int4(po, 70))
    assert np.array_equal(to_np(skinny.dequantize("int4", packed, scale, zero)), skinny_ref.dequantize("int4", po, so, zo))


@pytest.mark.parametrize("n,rows", [(32, 32), (37, 32), (5, 16), (64, 16)])
def test_int4_pack_round_trip(n, rows):
    q = torch.randint(0, 16, (n, 384), dtype=torch.uint8)
    packed = skinny.pack_int4(q, rows)
    assert packed.shape == (-(-n // rows), 3, rows, 64) and packed.dtype == torch.uint8
    assert torch.equal(skinny.unpack_int4(packed, n), q)
    # byte j of a group holds code j (low nibble) and code j + 64 (high nibble)
    assert int(packed[0, 1, 0, 5]) == int(q[0, 128 + 5]) | (int(q[0, 128 + 64 + 5]) << 4)


def test_int4_quantization_error_is_at_most_half_a_step():
    w = (torch.randn(24, 256) * 0.05).to(torch.bfloat16)
    packed, scale, zero = skinny.quantize_int4(w)
    assert scale.shape == zero.shape == (2, 24)
    deq = skinny.dequantize("int4", packed, scale, zero)
    step = scale.float().t().repeat_interleave(128, dim=1)
    assert ((deq - w.float()).abs() <= 0.55 * step + 1e-3).all()
    assert skinny.unpack_int4(packed, 24).max() <= 15
    with pytest.raises(ValueError):
        skinny.quantize_int4(torch.zeros(4, 100, dtype=torch.bfloat16))


def test_rowwise_quantization_error_bound():
    w = torch.randn(16, 256, dtype=torch.bfloat16)
    q, s = quantize_rowwise_int8(w)
    assert q.abs().max() <= 127
    deq = q.float() * s.float()[:, None]
    assert ((deq - w.float()).abs().amax(1) <= s.float() * 0.51 + 1e-3).all()


def test_skinny_mm_validation_matches_the_reference_errors():
    w = torch.zeros(8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        skinny.skinny_mm(torch.zeros(2, 64, dtype=torch.bfloat16), w)  # K mismatch
    with pytest.raises(ValueError):
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16)[:, ::2], w)  # not contiguous
    with pytest.raises(ValueError):
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16), torch.zeros(8, 128, dtype=torch.int8))  # no scale
    with pytest.raises(ValueError):
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16), torch.zeros(8, 128, dtype=torch.float16))
    with pytest.raises(ValueError):  # int4 without scale / zero
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16), torch.zeros(1, 1, 32, 64, dtype=torch.uint8))
    packed, sc, z = skinny.quantize_int4(torch.zeros(8, 256, dtype=torch.bfloat16))
    with pytest.raises(ValueError):  # K does not match the packed groups
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16), packed, sc, z)
    with pytest.raises(ValueError):  # scale with the wrong group count
        skinny.skinny_mm(torch.zeros(2, 256, dtype=torch.bfloat16), packed, sc[:1], z[:1])


def test_skinny_mm_empty_shapes_need_no_device():
    w = torch.zeros(8, 128, dtype=torch.bfloat16)
    assert skinny.skinny_mm(torch.zeros(0, 128, dtype=torch.bfloat16), w).shape == (0, 8)
    y = skinny.skinny_mm(torch.zeros(3, 0, dtype=torch.bfloat16), torch.zeros(8, 0, dtype=torch.bfloat16))
    assert y.shape == (3, 8) and (y == 0).all()


def test_cpu_tensors_are_refused():
    w = torch.zeros(8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        skinny.skinny_mm(torch.zeros(2, 128, dtype=torch.bfloat16), w)
    q, s = quantize_rowwise_int8(w)
    with pytest.raises(ValueError, match="CUDA"):
        gemv_int8(torch.zeros(1, 128, dtype=torch.bfloat16), q, s)
    lin = nn.Linear(128, 8, bias=False, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        SkinnyLinear(lin, "bf16_wo")(torch.zeros(1, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        Int8Linear(lin)(torch.zeros(1, 128, dtype=torch.bfloat16))


def test_skinny_linear_attributes_follow_the_reference():
    lin = nn.Linear(256, 64, bias=True, dtype=torch.bfloat16)
    a = SkinnyLinear(lin, "bf16_wo")
    assert a.weight is lin.weight and a.scale is None and a.bias is lin.bias
    b = SkinnyLinear(lin, "int8_wo")
    assert b.weight.numel() == 0 and b.weight.dtype == torch.bfloat16
    q, s = quantize_rowwise_int8(lin.weight.data)
    assert torch.equal(b.q, q) and torch.equal(b.scale, s)
    assert torch.equal(b.dequantized(torch.float32), q.float() * s.float()[:, None])
    assert b(torch.empty(0, 256, dtype=torch.bfloat16)).shape == (0, 64)
    with pytest.raises(ValueError):
        SkinnyLinear(lin, "fp8_wo")
    c = Int8Linear(lin)
    assert torch.equal(c.q, b.q) and torch.equal(c.scale, b.scale) and c.weight.numel() == 0


@pytest.mark.parametrize("name,target,want", [
    ("model.layers.3.self_attn.q_proj", "global", True),
    ("model.layers.3.mlp.down_proj", "all", True),
    ("model.layers.3.mlp.down_proj", "local", False),
    ("model.local_encoder.layers.0.xlstm.q", "local", True),
    ("model.local_encoder.layers.0.xlstm.igate_preact", "all", False),
    ("model.local_decoder.layers.2.mlp.up_proj", "local", True),
    ("model.local_encoder.out_projection", "local", True),
    ("model.local_decoder.in_projection", "all", True),
    ("model.local_encoder.boundary_predictor.0", "all", False),
    ("lm_head", "all", False),
    ("model.layers.3.self_attn.q_proj", "none", False),
])
def test_bolmo_selection(name, target, want):
    assert select.should_quantize(name, target) is want


def test_olmo_selection_and_errors():
    assert select.olmo_should_quantize("model.layers.0.mlp.gate_proj", "blocks")
    assert not select.olmo_should_quantize("lm_head", "blocks")
    assert select.olmo_should_quantize("lm_head", "blocks+head")
    assert not select.olmo_should_quantize("model.embed_tokens", "blocks+head")
    with pytest.raises(ValueError):
        select.should_quantize("x", "blocks")
    with pytest.raises(ValueError):
        select.olmo_should_quantize("x", "local")
    assert select.selects("all", "local") and not select.selects("blocks", "head")


class _Block(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.self_attn = nn.ModuleDict({n: nn.Linear(d, d, bias=False) for n in ("q_proj", "k_proj", "v_proj", "o_proj")})
        self.mlp = nn.ModuleDict({"gate_proj": nn.Linear(d, 2 * d, bias=False), "up_proj": nn.Linear(d, 2 * d, bias=False),
                                  "down_proj": nn.Linear(2 * d, d, bias=False)})


class _Toy(nn.Module):
    def __init__(self, d=64):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Block(d) for _ in range(2)])
        self.lm_head = nn.Linear(d, 32, bias=False)


@pytest.mark.parametrize("kernel,scheme,cls", [("skinny", "bf16_wo", SkinnyLinear), ("skinny", "int8_wo", SkinnyLinear),
                                               ("skinny", "int4_wo", SkinnyLinear), ("default", "int8_wo", Int8Linear)])
def test_apply_quantization_swaps_the_selected_linears(kernel, scheme, cls):
    m = _Toy(128 if scheme == "int4_wo" else 64).to(torch.bfloat16)  # int4 groups need K % 128 == 0
    stats = apply_quantization(m, "blocks", scheme, 128, None, None, kernel)
    assert stats["n_linears"] == 14
    assert ("kernel" in stats) == (kernel != "default")
    assert sum(isinstance(x, cls) for x in m.modules()) == 14
    assert isinstance(m.lm_head, nn.Linear)


def test_int4_skinny_linear_holds_the_packed_format():
    lin = nn.Linear(256, 40, bias=False).to(torch.bfloat16)
    sl = SkinnyLinear(lin, "int4_wo")
    packed, scale, zero = skinny.quantize_int4(lin.weight.data)
    assert torch.equal(sl.q, packed) and torch.equal(sl.scale, scale) and torch.equal(sl.zero, zero)
    assert sl.weight.numel() == 0 and sl.weight.dtype == torch.bfloat16
    assert torch.equal(sl.dequantized(torch.float32), skinny.dequantize("int4", packed, scale, zero))


def test_default_kernel_rejects_skinny_only_and_torchao_schemes():
    with pytest.raises(ValueError):
        apply_quantization(_Toy().to(torch.bfloat16), "blocks", "bf16_wo")
    with pytest.raises(NotImplementedError):
        apply_quantization(_Toy().to(torch.bfloat16), "blocks", "int4_wo")


def test_scan_geometry_limits():
    q = torch.zeros(3, 4, 96)
    v = torch.zeros(3, 4, 64)
    with pytest.raises(NotImplementedError):
        draft_fused._geometry(q, v)
    assert draft_fused._geometry(torch.zeros(3, 4, 512), torch.zeros(3, 4, 512)) == (4, 512, 512)
