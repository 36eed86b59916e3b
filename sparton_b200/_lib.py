"""ctypes binding of the native library (``include/sparton_b200.h``).

The library is built in-tree by ``sparton_b200.build`` into
``sparton_b200/_lib/libsparton_b200.so``. There is no fallback: if the library
is missing, or a call fails, a ``RuntimeError`` is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libsparton_b200.so")

# Status codes (sparton_status).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE = 5

# operand layouts of sparton_gemm
LAYOUT_ROWS = 0
LAYOUT_COLS = 1
# sparton_dtype
DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
# sparton_mask_dtype
MASK_DTYPE = {
    torch.bool: 0, torch.uint8: 0, torch.int32: 1, torch.int64: 2,
    torch.float32: 3, torch.float16: 4, torch.bfloat16: 5,
}

EXPORTED_SYMBOLS = (
    "sparton_abi_version",
    "sparton_last_error",
    "sparton_fwd_workspace_size",
    "sparton_fwd",
    "sparton_mask_prepare",
    "sparton_fwd_prepared",
    "sparton_fwd_noalloc",
    "sparton_fwd_noalloc_status",
    "sparton_bwd_workspace_size",
    "sparton_bwd",
    "sparton_reg_workspace_size",
    "sparton_reg_fwd",
    "sparton_reg_bwd",
    "sparton_sparse_workspace_size",
    "sparton_reps_csr",
    "sparton_reps_topk",
    "sparton_transform_fwd",
    "sparton_transform_workspace_size",
    "sparton_transform_bwd",
    "sparton_read_device_status",
    "sparton_selftest_wait_timeout",
    "sparton_gemm_workspace_size",
    "sparton_gemm",
    "sparton_pad_rows",
    "sparton_hidden_allreduce",
    "sparton_ipc_export",
    "sparton_ipc_open",
    "sparton_ipc_close",
)

_lock = threading.Lock()
_lib = None

_vp, _i, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t


def _declare(lib: ctypes.CDLL) -> None:
    lib.sparton_abi_version.argtypes = []
    lib.sparton_abi_version.restype = _i
    lib.sparton_last_error.argtypes = []
    lib.sparton_last_error.restype = ctypes.c_char_p
    lib.sparton_fwd_workspace_size.argtypes = [_i64] * 4
    lib.sparton_fwd_workspace_size.restype = _sz
    lib.sparton_bwd_workspace_size.argtypes = [_i64] * 4
    lib.sparton_bwd_workspace_size.restype = _sz
    lib.sparton_fwd.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i64, _i64, _i64, _i64,
                                _vp, _vp, _vp, _sz, _vp]
    lib.sparton_fwd.restype = _i
    lib.sparton_mask_prepare.argtypes = [_vp, _i, _i64, _i64, _vp, _sz, _vp]
    lib.sparton_mask_prepare.restype = _i
    lib.sparton_fwd_prepared.argtypes = [_vp, _vp, _vp, _i, _i64, _i64, _i64, _i64,
                                         _vp, _vp, _vp, _sz, _vp]
    lib.sparton_fwd_prepared.restype = _i
    lib.sparton_fwd_noalloc.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i64, _i64, _i64, _i64,
                                        _vp, _vp, _vp]
    lib.sparton_fwd_noalloc.restype = _i
    lib.sparton_fwd_noalloc_status.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint32)]
    lib.sparton_fwd_noalloc_status.restype = _i
    lib.sparton_bwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i64, _i64, _i64, _i64,
                                _vp, _vp, _vp, _i, _i, _vp, _sz, _vp]
    lib.sparton_bwd.restype = _i
    lib.sparton_reg_workspace_size.argtypes = [_i64, _i64]
    lib.sparton_reg_workspace_size.restype = _sz
    _f = ctypes.c_float
    lib.sparton_reg_fwd.argtypes = [_vp, _i, _i64, _i64, _f, _f, _vp, _vp, _vp, _sz, _vp]
    lib.sparton_reg_fwd.restype = _i
    lib.sparton_reg_bwd.argtypes = [_vp, _vp, _vp, _vp, _f, _f, _i, _i64, _i64, _vp, _vp]
    lib.sparton_reg_bwd.restype = _i
    lib.sparton_sparse_workspace_size.argtypes = [_i64, _i64]
    lib.sparton_sparse_workspace_size.restype = _sz
    lib.sparton_reps_csr.argtypes = [_vp, _i, _i64, _i64, _f, _vp, _vp, _vp, _i64, _vp, _sz, _vp]
    lib.sparton_reps_csr.restype = _i
    lib.sparton_reps_topk.argtypes = [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp]
    lib.sparton_reps_topk.restype = _i
    lib.sparton_transform_fwd.argtypes = [_vp, _vp, _vp, _f, _i, _i64, _i64, _vp, _vp, _vp, _vp]
    lib.sparton_transform_fwd.restype = _i
    lib.sparton_transform_workspace_size.argtypes = [_i64, _i64]
    lib.sparton_transform_workspace_size.restype = _sz
    lib.sparton_transform_bwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i64, _i64, _vp, _vp, _vp,
                                          _vp, _vp, _sz, _vp]
    lib.sparton_transform_bwd.restype = _i
    lib.sparton_read_device_status.argtypes = [_vp, _vp, ctypes.POINTER(ctypes.c_uint32)]
    lib.sparton_read_device_status.restype = _i
    lib.sparton_selftest_wait_timeout.argtypes = [ctypes.c_uint32, _vp, _sz, _vp]
    lib.sparton_selftest_wait_timeout.restype = _i
    lib.sparton_gemm_workspace_size.argtypes = [_i64, _i64, _i64]
    lib.sparton_gemm_workspace_size.restype = _sz
    lib.sparton_gemm.argtypes = [_vp, _i, _i64, _vp, _i, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i,
                                 _i64, _vp, _sz, _vp]
    lib.sparton_gemm.restype = _i
    lib.sparton_pad_rows.argtypes = [_vp, _i, _i64, _i64, _vp, _i64, _vp]
    lib.sparton_pad_rows.restype = _i
    lib.sparton_hidden_allreduce.argtypes = [_vp, _vp, _vp, _i, _i, ctypes.c_uint32, _vp, _i64,
                                             _i64, _i64, _vp, _i, _vp, _vp]
    lib.sparton_hidden_allreduce.restype = _i
    lib.sparton_ipc_export.argtypes = [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)]
    lib.sparton_ipc_export.restype = _i
    lib.sparton_ipc_open.argtypes = [_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
    lib.sparton_ipc_open.restype = _i
    lib.sparton_ipc_close.argtypes = [_vp, ctypes.c_uint64]
    lib.sparton_ipc_close.restype = _i


def load() -> ctypes.CDLL:
    """Loads (once) and returns the native library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"sparton_b200 native library not found at {LIB_PATH}; build it with "
                    "`python -m sparton_b200.build` (needs nvcc). There is no CPU fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            _declare(lib)
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().sparton_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int, what: str) -> None:
    """Raises the Python exception matching a sparton_status code."""
    if status == OK:
        return
    msg = f"{what} failed: {last_error()} (status {status})"
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_ZEROED: dict = {}


def zeroed_workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """A zero-filled device buffer of at least ``nbytes`` for the entry points
    whose workspace must be zero when a call starts and is left zero when it
    ends (sparton_reps_csr, sparton_reg_fwd): one per (device, current stream,
    tag), cleared once when allocated and reused by every later call on that
    stream."""
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream, tag)
    buf = _ZEROED.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _ZEROED[key] = buf
    return buf


def read_device_status(workspace: torch.Tensor) -> int:
    """Device status word of a forward workspace (0 = no device-side timeout)."""
    code = ctypes.c_uint32(0)
    with torch.cuda.device(workspace.device):
        check(load().sparton_read_device_status(ptr(workspace), stream_handle(workspace.device),
                                                ctypes.byref(code)),
              "sparton_read_device_status")
    return int(code.value)
