"""pytest setup: the `gpu` marker, the repo root on sys.path, and the in-tree kernel library.

Tests marked `gpu` need an sm_100 device; they fail (not skip) when selected without one, so a run
on a GPU box can never pass by skipping. Everything else runs on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


@pytest.fixture(scope="session", autouse=True)
def _kernel_library():
    """Builds libbp_kernels.so if a source is newer than it (no-op when the prebuilt library is current)."""
    from byteprof_b200 import build

    try:
        build.build()
    except RuntimeError:
        if not build.LIB_PATH.exists():
            raise
    yield


@pytest.fixture(autouse=True)
def _gpu_required(request):
    """GPU tests need a device, and no kernel may have raised a device error (a bounded wait that
    timed out) by the end of the test."""
    gpu = request.node.get_closest_marker("gpu") is not None
    if gpu:
        import torch

        assert torch.cuda.is_available(), "this test needs a CUDA device"
    yield
    if gpu:
        from byteprof_b200 import _lib

        assert _lib.device_errors() == 0, "a kernel reported a device error (bounded wait timed out)"
