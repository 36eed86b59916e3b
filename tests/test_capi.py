"""CPU checks of the C ABI: the library loads, exports every entry point that
include/sparton_b200.h declares, and rejects bad arguments before touching a
GPU. No compute is launched here."""
import ctypes
import os
import re

import pytest

from sparton_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "sparton_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sparton_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_header_declares_the_boundary():
    names = declared_functions()
    assert {"sparton_fwd", "sparton_bwd", "sparton_fwd_workspace_size",
            "sparton_bwd_workspace_size", "sparton_last_error"} <= set(names)
    assert sorted(_lib.EXPORTED_SYMBOLS) == names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.sparton_abi_version() == 1


def test_workspace_sizes(lib):
    B, S, D, V = 128, 256, 768, 30522
    fw = lib.sparton_fwd_workspace_size(B, S, D, V)
    assert fw >= 256 + 4 * B + 4 * B * (S // 32)
    bw = lib.sparton_bwd_workspace_size(B, S, D, V)
    assert bw >= 256 + 4 * B * (S + 1) + 2 * 8 * B * V  # offsets + two 8-byte record lists
    assert lib.sparton_fwd_workspace_size(-1, S, D, V) == 0


def _fwd(lib, B=2, S=8, D=16, V=10, ws=None, ws_size=None, dtype=2, mask_dtype=2):
    dummy = ctypes.c_void_p(0x1000)
    wsp = ctypes.c_void_p(0x100000) if ws is None else ws
    size = lib.sparton_fwd_workspace_size(B, S, D, V) if ws_size is None else ws_size
    return lib.sparton_fwd(dummy, dummy, None, dummy, mask_dtype, dtype, B, S, D, V, dummy, dummy,
                           wsp, size, None)


def test_rejects_negative_sizes(lib):
    assert _fwd(lib, B=-1) == _lib.ERR_INVALID_ARGUMENT
    assert "negative" in _lib.last_error()


def test_rejects_unaligned_hidden_size(lib):
    assert _fwd(lib, D=12) == _lib.ERR_UNSUPPORTED
    assert "multiple of 8" in _lib.last_error()


def test_rejects_small_workspace(lib):
    assert _fwd(lib, ws_size=16) == _lib.ERR_WORKSPACE
    assert "workspace" in _lib.last_error()


def test_rejects_unknown_dtypes(lib):
    assert _fwd(lib, dtype=7) == _lib.ERR_UNSUPPORTED
    assert _fwd(lib, mask_dtype=9) == _lib.ERR_UNSUPPORTED


def test_bwd_rejects_bad_grad_dtype(lib):
    dummy = ctypes.c_void_p(0x1000)
    B, S, D, V = 2, 8, 16, 10
    st = lib.sparton_bwd(dummy, dummy, dummy, dummy, dummy, 2, B, S, D, V, dummy, dummy, None,
                         1, 2, ctypes.c_void_p(0x100000), lib.sparton_bwd_workspace_size(B, S, D, V),
                         None)
    assert st == _lib.ERR_UNSUPPORTED


def test_valid_call_without_gpu_reports_device_error(lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _fwd(lib) == _lib.ERR_DEVICE
    assert "sm_100" in _lib.last_error()


def test_check_raises_python_errors():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")
    _lib.check(_lib.OK, "x")


def test_components_validate_before_any_launch(lib):
    """Argument checks of the entry points around the head run on the host,
    before any device access, so they answer without a GPU."""
    d = ctypes.c_void_p(0x1000)
    ws = ctypes.c_void_p(0x100000)
    # top-k: k outside [0, V], or above the 4096 the kernel sorts in shared memory
    assert lib.sparton_reps_topk(d, 2, 4, 100, 101, d, d, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_reps_topk(d, 2, 4, 10000, 4097, d, d, None) == _lib.ERR_UNSUPPORTED
    assert lib.sparton_reps_topk(d, 9, 4, 100, 5, d, d, None) == _lib.ERR_UNSUPPORTED  # dtype
    # CSR: no row pointers, negative capacity, capacity without outputs, small workspace
    wsz = lib.sparton_sparse_workspace_size(4, 100)
    assert lib.sparton_reps_csr(d, 2, 4, 100, 0.0, None, None, None, 0, ws, wsz, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_reps_csr(d, 2, 4, 100, 0.0, d, None, None, -1, ws, wsz, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_reps_csr(d, 2, 4, 100, 0.0, d, None, None, 10, ws, wsz, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_reps_csr(d, 2, 4, 100, 0.0, d, None, None, 0, ws, 4, None) == \
        _lib.ERR_WORKSPACE
    # transform: missing pointers, negative eps, too many rows for the parameter sums
    assert lib.sparton_transform_fwd(d, d, None, 1e-5, 2, 8, 16, d, d, d, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_transform_fwd(d, d, d, -1.0, 2, 8, 16, d, d, d, None) == \
        _lib.ERR_INVALID_ARGUMENT
    rows = 65535 * 256 + 1
    assert lib.sparton_transform_bwd(d, d, d, d, d, 2, rows, 16, d, d, None, None, ws,
                                     lib.sparton_transform_workspace_size(rows, 16), None) == \
        _lib.ERR_UNSUPPORTED
    # regularisers: small workspace
    assert lib.sparton_reg_fwd(d, 2, 4, 100, 1.0, 1.0, d, d, ws, 1, None) == _lib.ERR_WORKSPACE


def test_noalloc_checks_arguments_before_the_device(lib):
    """sparton_fwd_noalloc validates sizes, dtype and its scratch limit before
    it looks at the device (no GPU here): each is reported as itself."""
    dummy = ctypes.c_void_p(0x1000)
    assert lib.sparton_fwd_noalloc(dummy, dummy, None, dummy, 2, 2, -1, 8, 16, 10, dummy, dummy,
                                   None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_fwd_noalloc(dummy, dummy, None, dummy, 2, 7, 2, 8, 16, 10, dummy, dummy,
                                   None) == _lib.ERR_UNSUPPORTED
    assert "dtype" in _lib.last_error()
    assert lib.sparton_fwd_noalloc(dummy, dummy, None, dummy, 2, 2, 4096, 8192, 64, 100, dummy,
                                   dummy, None) == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
    assert lib.sparton_fwd_noalloc_status(None, None) == _lib.ERR_INVALID_ARGUMENT


def test_gemm_rejects_unaligned_operands(lib):
    """The tensor-core GEMM needs 16-byte operand rows (TMA): a K-major operand
    with K = 30522 (the vocabulary) is refused before any device work."""
    st = lib.sparton_gemm(None, 0, 0, None, 0, 0, None, 2, 128, 128, 30522, None, 0, 128, None, 0,
                          None)
    assert st == _lib.ERR_UNSUPPORTED and "multiple of 8" in _lib.last_error()
    assert lib.sparton_gemm(None, 0, 0, None, 0, 0, None, 0, 8, 8, 8, None, 0, 8, None, 0,
                            None) == _lib.ERR_UNSUPPORTED  # fp32 operands: no tensor-core kind
    assert lib.sparton_gemm(None, 0, 16, None, 0, 0, None, 2, 8, 8, 24, None, 0, 8, None, 0,
                            None) == _lib.ERR_INVALID_ARGUMENT  # lda below K
    assert lib.sparton_gemm_workspace_size(128, 128, 30528) > 128 * 128 * 4  # split-K partials
