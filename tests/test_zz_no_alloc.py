"""The entry point for callers that cannot allocate device memory, bp_skinny_mm_static_scratch.

Code running inside a CUDA-graph capture in global mode (where cudaMalloc is refused), or inside a host
application that gives its plugins no allocator, cannot hand bp_skinny_mm a workspace. This entry point
keeps the tensor-core path's scratch in a fixed array inside the library instead. Its results must be
those of bp_skinny_mm with a caller-provided workspace, call after call.

This file is collected last (test_zz_*), and it depends on no state left by other tests: it passes run
alone in a fresh process and after the rest of the suite.
"""

import pytest
import torch

from byteprof_b200 import _lib
from byteprof_b200.optim.skinny import skinny_mm
from helpers import deq_np, make_weights, to_np
from oracle import skinny_ref

pytestmark = pytest.mark.gpu


def _static_scratch_mm(x, w, out, scale=None):
    m, k = x.shape
    n = w.shape[0]
    with torch.cuda.device(x.device):
        _lib.call("bp_skinny_mm_static_scratch", x.data_ptr(), k, w.data_ptr(), _lib.dtype_code(w.dtype),
                  _lib.ptr(scale), out.data_ptr(), out.stride(0), _lib.dtype_code(out.dtype), m, n, k,
                  torch.cuda.current_stream(x.device).cuda_stream)
    return out


@pytest.mark.parametrize("kind", ["bf16", "int8"])
@pytest.mark.parametrize("n,k,m", [(100352, 2048, 4), (12288, 2048, 16), (2048, 2048, 1), (37, 256, 3)])
def test_static_scratch_matches_the_workspace_entry_point_twice_in_a_row(kind, n, k, m):
    """Large shapes (many tiles) use the static scratch for their stream-K partials; small ones need none.
    Two consecutive calls must both equal the result of the entry point with a caller workspace."""
    _, args = make_weights(kind, n, k, seed=31)
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    want = skinny_mm(x, *args)
    for _ in range(2):
        got = _static_scratch_mm(x, args[0], torch.empty(m, n, device="cuda", dtype=torch.bfloat16),
                                 args[1] if kind == "int8" else None)
        torch.cuda.synchronize()
        assert skinny_ref.nerr(to_np(got), to_np(x), deq_np(kind, args)) < skinny_ref.TOL_COMPONENTWISE
        assert torch.equal(got, want)
    assert _lib.device_errors() == 0


def test_static_scratch_entry_runs_inside_a_global_mode_graph_capture():
    """The use case it exists for: a stream captured in global mode, where allocation is refused. One call
    with a small shape (which needs no scratch) before the capture is the documented warm-up; the large bf16
    and int8 calls captured afterwards use the array and must not look anything up or allocate. Replayed
    twice, the graph gives the results of skinny_mm with a caller workspace."""
    dev = torch.device("cuda", torch.cuda.current_device())
    xs = torch.randn(3, 256, device=dev).to(torch.bfloat16)
    ws_small = torch.randn(37, 256, device=dev).to(torch.bfloat16)
    _static_scratch_mm(xs, ws_small, torch.empty(3, 37, device=dev, dtype=torch.bfloat16))
    cases = []
    for kind, n, k, m in (("bf16", 100352, 2048, 4), ("int8", 100352, 2048, 16)):
        _, args = make_weights(kind, n, k, seed=41)
        x = torch.randn(m, k, generator=torch.Generator(device=dev).manual_seed(9), device=dev).to(torch.bfloat16)
        want = skinny_mm(x, *args)  # loads the kernels this shape runs, outside the capture
        cases.append((x, args, torch.empty(m, n, device=dev, dtype=torch.bfloat16), want, kind))
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side, capture_error_mode="global"):
        for x, args, out, _, kind in cases:
            _static_scratch_mm(x, args[0], out, args[1] if kind == "int8" else None)
    for _ in range(2):
        for _, _, out, _, _ in cases:
            out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for _, _, out, want, kind in cases:
            assert torch.equal(out, want), kind
    del g
    assert _lib.device_errors() == 0


def test_static_scratch_rejects_problems_beyond_its_limit():
    x = torch.zeros(1, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 64, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(1, 8, device="cuda", dtype=torch.bfloat16)
    st = _lib.lib().bp_skinny_mm_static_scratch(x.data_ptr(), 64, w.data_ptr(), 0, None, y.data_ptr(), 8, 0, 1,
                                                2_000_000, 64, None)
    assert st == 2 and b"static scratch" in _lib.lib().bp_last_error()
