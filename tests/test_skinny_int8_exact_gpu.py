"""The int8 tensor-core path sums exactly: each activation row is written in fixed point 29 bits below its
largest exponent (every x within 2^-22 of the row maximum is exact), the integer sums are exact, and
y = fp32(sum * scale) is rounded once. So the fp32 output equals the float64 value of
scale[n] * sum_k q[n, k] x[m, k] rounded to fp32, does not depend on how the kernel split K, and rows of
x holding Inf or NaN give NaN rows. (The reference's fp32 tensor-core sum is within its own rounding of
the same value; the oracle tests bound both against it.)"""

import numpy as np
import pytest
import torch

from byteprof_b200.optim import skinny as S
from helpers import make_weights, to_np

pytestmark = pytest.mark.gpu


def x_rows(m, k, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(m, k, generator=g, device="cuda") * scale).to(torch.bfloat16)


def exact64(x, q, s):
    """scale[n] * sum_k q[n, k] x[m, k] in float64 (exact sums for these inputs: every product has at
    most 15 significant bits and the partial sums span fewer than 53 bits)."""
    acc = to_np(x).astype(np.float64) @ to_np(q).astype(np.float64).T
    return acc * to_np(s).astype(np.float64)[None, :]


def ulps_apart(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


@pytest.mark.parametrize("n,k", [(2048, 2048), (8192, 2048), (2048, 8192), (100352, 2048), (300, 2064), (50, 144),
                                 (1000, 16)])
@pytest.mark.parametrize("m", [1, 5, 16])
def test_fp32_output_is_the_correctly_rounded_exact_sum(n, k, m):
    _, (q, s) = make_weights("int8", n, k, seed=n + k)
    x = x_rows(m, k, seed=m + k)
    y = S.skinny_mm(x, q, s, out=torch.empty(m, n, device="cuda", dtype=torch.float32))
    want = exact64(x, q, s).astype(np.float32)
    d = ulps_apart(to_np(y), want)
    assert d.max() <= 1, d.max()
    assert np.mean(d == 0) >= 0.999


def test_bf16_output_is_the_fp32_result_rounded_to_nearest_even():
    _, (q, s) = make_weights("int8", 8192, 2048, seed=4)
    x = x_rows(9, 2048, seed=4)
    y32 = S.skinny_mm(x, q, s, out=torch.empty(9, 8192, device="cuda", dtype=torch.float32))
    assert torch.equal(S.skinny_mm(x, q, s), y32.to(torch.bfloat16))


@pytest.mark.parametrize("lo,hi", [(0, 4096), (5000, 9096), (99000, 100352)])
def test_a_row_of_y_depends_only_on_its_weight_row(lo, hi):
    """Different N give different stream-K splits; the exact sums make the shared rows bit-identical."""
    _, (q, s) = make_weights("int8", 100352, 2048, seed=8)
    x = x_rows(16, 2048, seed=8)
    full = S.skinny_mm(x, q, s)
    part = S.skinny_mm(x, q[lo:hi], s[lo:hi])
    assert torch.equal(full[:, lo:hi], part)


def test_rows_with_inf_or_nan_give_nan_rows_and_leave_the_others_alone():
    _, (q, s) = make_weights("int8", 4096, 2048, seed=2)
    x = x_rows(6, 2048, seed=2)
    clean = S.skinny_mm(x, q, s)
    bad = x.clone()
    bad[1, 7] = float("inf")
    bad[4, 2000] = float("nan")
    y = S.skinny_mm(bad, q, s)
    assert torch.isnan(y[1]).all() and torch.isnan(y[4]).all()
    keep = [0, 2, 3, 5]
    assert torch.equal(y[keep], clean[keep])


def test_wide_dynamic_range_stays_within_the_fixed_point_bound():
    """Values far below the row maximum are rounded to the row's fixed-point unit 2^(e - 29): the error
    is at most half a unit per element, i.e. sum_k |q| * 2^(e - 30) * |scale| per output."""
    n, k, m = 1024, 2048, 4
    _, (q, s) = make_weights("int8", n, k, seed=6)
    g = torch.Generator(device="cuda").manual_seed(6)
    mag = torch.exp2(torch.randint(-60, 8, (m, k), generator=g, device="cuda").float())
    x = (torch.randn(m, k, generator=g, device="cuda") * mag).to(torch.bfloat16)
    y = to_np(S.skinny_mm(x, q, s, out=torch.empty(m, n, device="cuda", dtype=torch.float32))).astype(np.float64)
    want = exact64(x, q, s)
    xn = to_np(x).astype(np.float64)
    e = np.floor(np.log2(np.abs(xn).max(axis=1)))
    bound = (np.abs(to_np(q)).astype(np.float64).sum(axis=1)[None, :] * np.abs(to_np(s))[None, :] *
             np.exp2(e - 30)[:, None])
    assert (np.abs(y - want) <= bound + np.abs(want) * 2.0**-23 + 1e-30).all()


def test_zero_and_subnormal_rows():
    n, k = 512, 1024
    _, (q, s) = make_weights("int8", n, k, seed=9)
    x = x_rows(3, k, seed=9)
    x[0] = 0
    x[1] = (torch.randn(k, device="cuda") * 1e-39).to(torch.bfloat16)  # bf16 subnormals (and zeros)
    y = S.skinny_mm(x, q, s, out=torch.empty(3, n, device="cuda", dtype=torch.float32))
    assert (to_np(y[0]) == 0).all()
    want = exact64(x, q, s).astype(np.float32)
    assert ulps_apart(to_np(y[1:]), want[1:]).max() <= 1


def test_int8_stream_k_leaves_the_workspace_clean_and_repeats_bitwise():
    from byteprof_b200 import _lib

    _, (q, s) = make_weights("int8", 100352, 2048, seed=12)
    x = x_rows(16, 2048, seed=12)
    first = S.skinny_mm(x, q, s)
    for _ in range(3):
        assert torch.equal(S.skinny_mm(x, q, s), first)
    torch.cuda.synchronize()
    ws = _lib._workspaces[torch.cuda.current_device()]
    assert int(ws[:4 * 8192].view(torch.int32).abs().sum()) == 0


def _with_path(path, fn):
    import os

    old = os.environ.get("BP_SKINNY_PATH")
    os.environ["BP_SKINNY_PATH"] = path
    try:
        out = fn()
        torch.cuda.synchronize()
        return out
    finally:
        if old is None:
            del os.environ["BP_SKINNY_PATH"]
        else:
            os.environ["BP_SKINNY_PATH"] = old


@pytest.mark.parametrize("n,k", [(2048, 2048), (8192, 2048), (2048, 8192), (100352, 2048), (300, 2064), (50, 144),
                                 (1000, 16), (37, 65536)])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_cuda_core_exact_kernel_gives_the_tensor_core_bits(n, k, m, out_dtype):
    """The exact CUDA-core int8 kernel (M <= 4) and the tensor-core kernel form the same integer sums from
    the same fixed-point digits and round once the same way: their outputs are bit-identical, so routing
    between them by M never changes a row's result."""
    _, (q, s) = make_weights("int8", n, k, seed=n + k)
    x = x_rows(m, k, seed=m, scale=3.0)
    x[0, 5] = 1e-30  # tiny values far below the row maximum round in the fixed point, the same in both
    run = lambda: S.skinny_mm(x, q, s, out=torch.empty(m, n, device="cuda", dtype=out_dtype))  # noqa: E731
    tc = _with_path("tc", run)
    ex = _with_path("exact", run)
    assert torch.equal(tc, ex)
    assert torch.equal(S.skinny_mm(x, q, s, out=torch.empty(m, n, device="cuda", dtype=out_dtype)), ex)  # default route


def test_cuda_core_exact_kernel_nan_rows_and_zero_rows():
    _, (q, s) = make_weights("int8", 2048, 2048, seed=1)
    x = x_rows(4, 2048, seed=2)
    x[1, 7] = float("inf")
    x[2].zero_()
    x[3, 100] = float("nan")
    y = _with_path("exact", lambda: S.skinny_mm(x, q, s, out=torch.empty(4, 2048, device="cuda")))
    assert torch.isnan(y[1]).all() and torch.isnan(y[3]).all()
    assert (y[2] == 0).all() and torch.isfinite(y[0]).all()
    tc = _with_path("tc", lambda: S.skinny_mm(x, q, s, out=torch.empty(4, 2048, device="cuda")))
    assert torch.equal(torch.nan_to_num(tc, nan=7.0), torch.nan_to_num(y, nan=7.0))
