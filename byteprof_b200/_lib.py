"""ctypes binding of the C ABI in `include/bp_kernels.h` (libbp_kernels.so, built in-tree).

The library is loaded once per process. A missing library or a non-zero status raises: there is no
fallback path. Every call passes torch's current CUDA stream of the tensor's device, so launches
are ordered with the surrounding torch work and can be captured in CUDA graphs.
"""

from __future__ import annotations

import contextlib
import ctypes
from ctypes import c_float, c_int, c_longlong, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libbp_kernels.so"

BP_OK = 0
BP_DTYPE_BF16, BP_DTYPE_F32, BP_DTYPE_INT8, BP_DTYPE_INT4 = 0, 1, 2, 3
_DTYPE_CODE = {torch.bfloat16: BP_DTYPE_BF16, torch.float32: BP_DTYPE_F32, torch.int8: BP_DTYPE_INT8}

# name -> (restype, argtypes); must match include/bp_kernels.h
_SIGNATURES = {
    "bp_abi_version": (c_int, []),
    "bp_status_string": (ctypes.c_char_p, [c_int]),
    "bp_last_error": (ctypes.c_char_p, []),
    "bp_skinny_mm": (c_int, [c_void_p, c_longlong, c_void_p, c_int, c_void_p, c_void_p, c_longlong, c_int,
                             c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bp_skinny_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "bp_skinny_mm_static_scratch": (c_int, [c_void_p, c_longlong, c_void_p, c_int, c_void_p, c_void_p, c_longlong,
                                            c_int, c_int, c_int, c_int, c_void_p]),
    "bp_skinny_mm_xf32": (c_int, [c_void_p, c_longlong, c_void_p, c_int, c_void_p, c_void_p, c_longlong, c_int,
                                  c_int, c_int, c_int, c_void_p]),
    "bp_gemv_int8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t,
                             c_void_p]),
    "bp_skinny_mm_int4": (c_int, [c_void_p, c_longlong, c_void_p, c_void_p, c_void_p, c_void_p, c_longlong, c_int,
                                  c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bp_rmsnorm": (c_int, [c_void_p, c_longlong, c_void_p, c_void_p, c_longlong, c_int, c_int, c_float, c_void_p]),
    "bp_rmsnorm_ex": (c_int, [c_void_p, c_longlong, c_void_p, c_int, c_void_p, c_longlong, c_void_p, c_longlong,
                              c_void_p, c_longlong, c_int, c_int, c_float, c_int, c_int, c_void_p]),
    "bp_decode_loop": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_longlong, c_int, c_int,
                               c_void_p, c_void_p, c_void_p, c_void_p]),
    "bp_embed_rmsnorm": (c_int, [c_void_p, c_longlong, c_longlong, c_void_p, c_void_p, c_void_p, c_longlong,
                                 c_void_p, c_longlong, c_int, c_int, c_float, c_void_p]),
    "bp_swiglu": (c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_int, c_int, c_void_p]),
    "bp_gate_softcap": (c_int, [c_void_p, c_longlong, c_void_p, c_void_p, c_longlong, c_int, c_int, c_float,
                                c_void_p]),
    "bp_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int, c_int, c_int, c_float, c_float, c_int, c_void_p]),
    "bp_decode_finish": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "bp_glob_step_workspace_bytes": (c_size_t, []),
    "bp_loc_step_workspace_bytes": (c_size_t, []),
    "bp_loc_enc_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_float, c_float, c_float, c_void_p, c_size_t, c_void_p]),
    "bp_loc_dec_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_float, c_float, c_float, c_void_p, c_size_t, c_void_p]),
    "bp_loc_encdec_step": (c_int, [c_void_p] * 16 + [c_float, c_float, c_float, c_void_p, c_size_t, c_void_p]),
    "bp_glob_step": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float,
                             c_void_p, c_size_t, c_void_p]),
    "bp_mlstm_scan": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_int, c_int, c_int, c_int, c_longlong, c_longlong, c_longlong, c_longlong,
                              c_int, c_int, c_float, c_float, c_void_p]),
    "bp_mlstm_accept": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "bp_mlstm_commit_state": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_longlong,
                                      c_longlong, c_longlong, c_void_p, c_int, c_int, c_void_p]),
    "bp_device_errors": (c_int, [ctypes.POINTER(ctypes.c_uint)]),
}

_lib: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A kernel entry point returned a non-zero status."""

    def __init__(self, name: str, status: int, message: str):
        super().__init__(f"{name}: {message or 'status ' + str(status)} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built (`python -m byteprof_b200.build`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m byteprof_b200.build` "
                               "(there is no fallback implementation)")
        cdll = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(cdll, name)
            fn.restype = res
            fn.argtypes = args
        _lib = cdll
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


_fns: dict[str, object] = {}


def call(name: str, *args) -> None:
    """Calls an entry point and raises KernelError on a non-zero status."""
    fn = _fns.get(name)
    if fn is None:
        fn = getattr(lib(), name)
        _fns[name] = fn
    st = fn(*args)
    if st != BP_OK:
        msg = lib().bp_last_error().decode(errors="replace")
        raise KernelError(name, st, msg)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """torch's current stream on the tensor's device, as a raw cudaStream_t (torch's own raw query when
    it has one: a Stream object costs more host time than the launch it is for)."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


_NO_SWITCH = contextlib.nullcontext()


def on_device(t: torch.Tensor):
    """torch.cuda.device(t.device), or nothing when that device is already current (the usual case;
    entering and leaving the context costs a few microseconds of host time per call)."""
    if t.device.index == torch.cuda.current_device():
        return _NO_SWITCH
    return torch.cuda.device(t.device)


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("the byteprof B200 kernels take CUDA tensors only (there is no CPU path)")


# ---- skinny workspace --------------------------------------------------------------------------------
# One zero-filled scratch buffer per device for the stream-K partial sums of the tensor-core paths
# (about 9.5 MB for int8 weights on 148 SMs). Kernels leave it zero-filled. Calls that overlap in time on
# different streams of one device would share it, which the C ABI forbids: the operator API serialises
# on torch's current stream.
WORKSPACE_CAPACITY = 16 << 20
_workspaces: dict[int, torch.Tensor] = {}
_ws_need: dict[tuple[int, int, int, int], int] = {}


def skinny_workspace(device: torch.device, m: int, n: int, k: int, w_dtype: int) -> tuple[int | None, int]:
    """(pointer, bytes) of the device's skinny workspace, large enough for this problem."""
    key = (device.index, n, k, w_dtype)
    need = _ws_need.get(key)
    if need is None:
        need = int(lib().bp_skinny_workspace_bytes(min(m, 16), n, k, w_dtype))
        _ws_need[key] = need
    if need == 0:
        return None, 0
    ws = _workspaces.get(device.index)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the skinny workspace is allocated on the first call: run one call outside CUDA-graph "
                               "capture first (the usual warm-up)")
        ws = torch.zeros(max(WORKSPACE_CAPACITY, need), dtype=torch.uint8, device=device)
        _workspaces[device.index] = ws
    return ws.data_ptr(), ws.numel()


def device_errors() -> int:
    """Error flags the kernels raised on the current device since the last call (then cleared)."""
    v = ctypes.c_uint(0)
    call("bp_device_errors", ctypes.byref(v))
    return int(v.value)
