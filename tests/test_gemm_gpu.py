"""The tensor-core GEMM (sparton_gemm) against a plain torch fp32 reference of
the same product, through the C ABI: both operand layouts for A and B, output
tiles with ragged edges (M, N not multiples of 128 / 256, K not a multiple of
64), K split over several units (long contractions over few tiles), bias, and
bf16 / f16 / fp32 outputs.

Tolerance: the operands are the same 16-bit values on both sides and the sums
are fp32 on both, so only the summation order differs: |C - ref| <= 1e-3 *
sum_k |A B| for an fp32 C, plus one rounding of the output type (2^-8 relative
for bf16, 2^-11 for f16) for a 16-bit C.
"""
import pytest
import torch

from sparton_b200 import _lib

pytestmark = pytest.mark.gpu

OUT_RTOL = {torch.float32: 0.0, torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}


def run_gemm(A, a_cols, B, b_cols, bias=None, out_dtype=None):
    """A: [M,K] (a_cols: stored as A.T contiguous [K,M]); B: [N,K] likewise."""
    lib = _lib.load()
    M, K = A.shape
    N = B.shape[0]
    dt = A.dtype
    out_dtype = out_dtype or dt
    a_mem = A.t().contiguous() if a_cols else A.contiguous()
    b_mem = B.t().contiguous() if b_cols else B.contiguous()
    C = torch.empty(M, N, dtype=out_dtype, device=A.device)
    ws = torch.empty(lib.sparton_gemm_workspace_size(M, N, K), dtype=torch.uint8, device=A.device)
    st = lib.sparton_gemm(a_mem.data_ptr(), int(a_cols), 0, b_mem.data_ptr(), int(b_cols), 0,
                          _lib.ptr(bias), _lib.DTYPE[dt], M, N, K, C.data_ptr(),
                          _lib.DTYPE[out_dtype], N, ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "sparton_gemm")
    assert _lib.read_device_status(ws) == 0
    return C


def check(C, A, B, bias):
    ref = A.float() @ B.float().t()
    mag = A.float().abs() @ B.float().abs().t()
    if bias is not None:
        ref = ref + bias.float()
        mag = mag + bias.float().abs()
    err = (C.float() - ref).abs()
    allowed = 1e-3 * mag + OUT_RTOL[C.dtype] * ref.abs() + 1e-6
    bad = err > allowed
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} off, worst {float((err - allowed).max()):.3g}"


SHAPES = [
    # M, N, K
    (128, 256, 64),
    (296, 200, 136),       # ragged M, N, K
    (64, 40, 72),          # one partial tile
    (768, 768, 4096),      # split K (few tiles, long K)
    (128, 128, 30528),     # InfoNCE-like: one tile, very long K
    (1000, 768, 768),      # transform-like
]


@pytest.mark.parametrize("layouts", [(False, False), (False, True), (True, False), (True, True)],
                         ids=["rows_rows", "rows_cols", "cols_rows", "cols_cols"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "M{}N{}K{}".format(*s))
def test_gemm_layouts_and_shapes(layouts, shape):
    M, N, K = shape
    a_cols, b_cols = layouts
    gen = torch.Generator().manual_seed(M + N + K)
    A = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    B = torch.randn(N, K, generator=gen).to(torch.bfloat16).cuda()
    C = run_gemm(A, a_cols, B, b_cols, out_dtype=torch.float32)
    torch.cuda.synchronize()
    check(C, A, B, None)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out", ["same", "f32"])
def test_gemm_bias_and_output_types(dtype, out):
    M, N, K = 333, 520, 256
    gen = torch.Generator().manual_seed(3)
    A = torch.randn(M, K, generator=gen).to(dtype).cuda()
    B = (torch.randn(N, K, generator=gen) * 0.1).to(dtype).cuda()
    bias = torch.randn(N, generator=gen).to(dtype).cuda()
    out_dtype = dtype if out == "same" else torch.float32
    C = run_gemm(A, False, B, False, bias=bias, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert C.dtype == out_dtype
    check(C, A, B, bias)


def test_gemm_split_k_with_bias_is_deterministic():
    M, N, K = 256, 256, 8192  # few tiles, long K: split over the K range
    gen = torch.Generator().manual_seed(5)
    A = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    B = torch.randn(N, K, generator=gen).to(torch.bfloat16).cuda()
    bias = torch.randn(N, generator=gen).to(torch.bfloat16).cuda()
    C1 = run_gemm(A, True, B, True, bias=bias, out_dtype=torch.float32)
    C2 = run_gemm(A, True, B, True, bias=bias, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    check(C1, A, B, bias)



@pytest.mark.parametrize("b_t", [False, True])
def test_gemm_padded_operands_and_unaligned_output(b_t):
    """Operands given as row-contiguous views of zero-padded buffers (rows of a
    multiple of 8 elements, as sparton_pad_rows makes them) and an output whose
    rows (N = 2999 elements) are not 16-byte aligned, stored through the
    epilogue's staging tile."""
    from sparton_b200.gemm import gemm, padded

    M, N, K = 200, 2999, 130
    gen = torch.Generator().manual_seed(9)
    A = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    B = torch.randn(N, K, generator=gen).to(torch.bfloat16).cuda()
    a = padded(A, 8)                      # [M, K] view, rows of 136
    b = padded(B.t(), 8) if b_t else padded(B, 8)
    assert a.stride(0) == 136 and not a.is_contiguous()
    C = gemm(a, b, b_t=b_t)
    torch.cuda.synchronize()
    assert C.shape == (M, N) and C.is_contiguous()
    check(C, A, B, None)


def test_pad_rows_zero_fills():
    from sparton_b200.gemm import padded

    x = torch.randn(37, 2999, dtype=torch.float16, device="cuda")
    v = padded(x, 64)
    torch.cuda.synchronize()
    assert v.stride(0) == 3008 and torch.equal(v, x)
    full = torch.as_strided(v, (37, 3008), (3008, 1))
    assert (full[:, 2999:] == 0).all()


def test_gemm_wide_output_picks_balanced_tiles():
    """M = 32768 rows x N = 768 (the transform's dense layer): enough tiles for
    several rounds over the SMs, so the kernel picks a narrower tile width; the
    result is the same product."""
    M, N, K = 32768, 768, 768
    gen = torch.Generator().manual_seed(11)
    A = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    B = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    bias = torch.randn(N, generator=gen).to(torch.bfloat16).cuda()
    C = run_gemm(A, False, B, False, bias=bias)
    torch.cuda.synchronize()
    check(C[:4096], A[:4096], B, bias)
    check(C[-4096:], A[-4096:], B, bias)
