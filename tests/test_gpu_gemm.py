"""tcgen05 GEMM parity against a plain PyTorch fp32 GEMM of the same bf16 operands.

Covers all four operand majors (K-major / MN-major for A and B), ragged
M/N/K (tile tails, TMA zero fill), split-K weight-grad shapes, bf16 output
and alpha/beta accumulation, i.e. every form in which the grafted MLP step
calls the kernel (forward x.W^T, input grad dy.W, weight grad X^T.dY).
"""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib

pytestmark = pytest.mark.gpu


def _operand(rows, k, mn_major, gen):
    """Returns (logical [rows,K] fp32 copy, storage tensor, ld)."""
    if not mn_major:
        ld = (k + 7) // 8 * 8 + 8
        store = torch.randn(rows, ld, generator=gen, device="cuda").to(torch.bfloat16)
        logical = store[:, :k]
    else:
        ld = (rows + 7) // 8 * 8 + 8
        store = torch.randn(k, ld, generator=gen, device="cuda").to(torch.bfloat16)
        logical = store[:, :rows].t()
    return logical.float(), store, ld


def run_gemm(A, lda, a_mn, B, ldb, b_mn, Cm, ldc, c_dtype, M, N, K, alpha=1.0, beta=0.0):
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("glt_gemm", C.c_void_p(A.data_ptr()), lda, a_mn, C.c_void_p(B.data_ptr()), ldb,
              b_mn, C.c_void_p(Cm.data_ptr()), ldc, c_dtype, M, N, K, alpha, beta, C.c_void_p(s))


CASES = [
    # M, N, K
    (128, 128, 64),
    (256, 512, 256),
    (384, 2048, 320),      # BN=256 path
    (300, 520, 200),       # ragged tails everywhere
    (128, 256, 8192),      # split-K (few tiles, long K)
    (1024, 4096, 1024),
]


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", CASES)
def test_gemm_f32_out(a_mn, b_mn, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K + a_mn * 2 + b_mn)
    a_log, a_st, lda = _operand(M, K, a_mn, g)
    b_log, b_st, ldb = _operand(N, K, b_mn, g)
    ldc = (N + 7) // 8 * 8
    out = torch.full((M, ldc), float("nan"), device="cuda")
    run_gemm(a_st, lda, a_mn, b_st, ldb, b_mn, out, ldc, 0, M, N, K)
    torch.cuda.synchronize()
    ref = a_log @ b_log.t()
    torch.testing.assert_close(out[:, :N], ref, rtol=2e-3, atol=2e-3 * K ** 0.5)


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1)])
def test_gemm_bf16_out(a_mn, b_mn):
    M, N, K = 512, 4096, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    a_log, a_st, lda = _operand(M, K, a_mn, g)
    b_log, b_st, ldb = _operand(N, K, b_mn, g)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    run_gemm(a_st, lda, a_mn, b_st, ldb, b_mn, out, N, 1, M, N, K)
    torch.cuda.synchronize()
    ref = (a_log @ b_log.t()).to(torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)


def test_gemm_alpha_beta():
    M, N, K = 256, 384, 192
    g = torch.Generator(device="cuda").manual_seed(5)
    a_log, a_st, lda = _operand(M, K, 0, g)
    b_log, b_st, ldb = _operand(N, K, 0, g)
    base = torch.randn(M, N, generator=g, device="cuda")
    out = base.clone()
    run_gemm(a_st, lda, 0, b_st, ldb, 0, out, N, 0, M, N, K, alpha=0.5, beta=1.0)
    torch.cuda.synchronize()
    ref = 0.5 * (a_log @ b_log.t()) + base
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-2)


def test_device_error_word_clear():
    code = C.c_uint(123)
    _lib.call("glt_device_error", C.byref(code))
    assert code.value == 0
