"""The C-ABI library loads on the CPU and exports every symbol include/bp_kernels.h declares; the
argument checks that run before any device work return their status codes (no kernel is launched)."""

import ctypes
import re
from pathlib import Path

import pytest

from byteprof_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "bp_kernels.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^\s*(?:int|size_t|const char\*)\s+(bp_\w+)\s*\(", text, re.M)


def test_header_and_binding_agree():
    names = declared_functions()
    assert names, "no declarations found"
    assert set(names) == set(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    cdll = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(cdll, name), name


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.bp_abi_version() == 205
    assert L.bp_status_string(0) == b"ok"
    assert L.bp_status_string(3) == b"misaligned"
    assert L.bp_status_string(99) == b"unknown status"


def test_status_codes_match_the_header():
    text = HEADER.read_text()
    codes = dict(re.findall(r"(BP_\w+) = (\d+)", text))
    assert int(codes["BP_OK"]) == _lib.BP_OK
    assert int(codes["BP_DTYPE_BF16"]) == _lib.BP_DTYPE_BF16
    assert int(codes["BP_DTYPE_F32"]) == _lib.BP_DTYPE_F32
    assert int(codes["BP_DTYPE_INT8"]) == _lib.BP_DTYPE_INT8


@pytest.mark.parametrize("args,msg", [
    ((None, 0, None, 0, None, None, 0, 0, -1, 4, 4, None, 0, None), b"negative size"),
    ((None, 0, None, 7, None, None, 0, 0, 1, 4, 4, None, 0, None), b"weight dtype"),
    ((None, 0, None, 0, None, None, 0, 5, 1, 4, 4, None, 0, None), b"output dtype"),
    ((None, 0, None, 0, None, None, 4, 0, 4, 4, 4, None, 0, None), b"y is NULL"),
])
def test_skinny_rejects_bad_arguments_before_touching_a_device(args, msg):
    L = _lib.lib()
    assert L.bp_skinny_mm(*args) == 1
    assert msg in L.bp_last_error()


def test_empty_problems_return_ok_without_a_device():
    L = _lib.lib()
    assert L.bp_skinny_mm(None, 0, None, 0, None, None, 0, 0, 0, 4, 4, None, 0, None) == 0
    assert L.bp_skinny_mm(None, 0, None, 0, None, None, 0, 0, 3, 0, 4, None, 0, None) == 0
    assert L.bp_last_error() == b""


def test_scan_rejects_unsupported_geometry_and_aliasing():
    L = _lib.lib()
    z = ctypes.c_void_p(16)
    base = [z, z, z, z, z, z, z, z, None, None, None, None, None, None, None]
    sizes = [4, 2, 64, 48, 256, 96, 2, 96, 0, 0, 1.0, 1e-6, None]
    st = L.bp_mlstm_scan(*base, 4, 2, 64, 40, 128, 80, 2, 80, 0, 0, 1.0, 1e-6, None)  # DV % 16 != 0
    assert st == 2 and b"DV" in L.bp_last_error()
    alias = list(base)
    alias[10] = z  # n_out == n_in
    st = L.bp_mlstm_scan(*alias, *sizes)
    assert st == 1 and b"alias" in L.bp_last_error()
    st = L.bp_mlstm_scan(*base, 4, 2, 64, 48, 250, 96, 2, 96, 0, 0, 1.0, 1e-6, None)  # q stride not a multiple of 8
    assert st == 3


def test_accept_rejects_bad_sizes():
    L = _lib.lib()
    assert L.bp_mlstm_accept(None, None, None, 5, 3, None) == 1


def test_workspace_query_without_a_device():
    L = _lib.lib()
    assert L.bp_skinny_workspace_bytes(4, 2048, 2048, 0) == 0  # bf16, few tiles: cluster split-K, no workspace
    assert L.bp_skinny_workspace_bytes(4, 2048, 2048, 2) > 0   # int8: stream-K, exact int64 partials
    assert L.bp_skinny_workspace_bytes(4, 100352, 2048, 2) <= 16 << 20  # fits the operator API's buffer
    assert L.bp_skinny_workspace_bytes(0, 2048, 2048, 0) == 0
    assert L.bp_skinny_workspace_bytes(4, 0, 2048, 0) == 0


def test_binding_argument_counts_match_the_header():
    text = HEADER.read_text()
    for name, (_, args) in _lib._SIGNATURES.items():
        decl = re.search(r"\b" + name + r"\s*\(([^;]*)\);", text, re.S).group(1).strip()
        n = 0 if decl in ("void", "") else decl.count(",") + 1
        assert n == len(args), name
