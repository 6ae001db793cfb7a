"""Two-SM (cta_group::2) GEMM tiles against a plain PyTorch fp32 GEMM and
against the one-SM kernel on the same bf16 operands.

glt_gemm_pair_mode(1) makes every 256-column GEMM of the library run on CTA
pairs (256 x 256 tiles, 128 rows of A and of B staged per CTA); glt_gemm
takes that path for N >= 2048.  Covers the four operand majors, ragged M/N/K
(a pair whose second CTA's rows are all past M, N not a multiple of 256,
K not a multiple of 64), more tiles than resident pairs (the persistent loop
over both accumulators and every ring phase), bf16 output and
alpha/beta accumulation.
"""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib
from tests.test_gpu_gemm import _operand, run_gemm

pytestmark = pytest.mark.gpu

CASES = [
    # M, N, K
    (384, 2048, 320),
    (300, 2600, 200),     # ragged everywhere
    (100, 2048, 64),      # one pair, second CTA entirely past M
    (1024, 4096, 1024),
    (4096, 6144, 2048),   # 384 tiles over at most 74 pairs
]


@pytest.fixture
def pair_mode():
    prev = _lib.lib.glt_gemm_pair_mode(-1)
    assert _lib.lib.glt_gemm_pair_mode(1) == 1
    yield
    _lib.lib.glt_gemm_pair_mode(prev)


def _gemm(a_st, lda, a_mn, b_st, ldb, b_mn, M, N, K, pair, c_dtype=0, alpha=1.0, beta=0.0, base=None):
    _lib.lib.glt_gemm_pair_mode(1 if pair else 0)
    ldc = (N + 7) // 8 * 8
    if base is not None:
        out = base.clone()
    elif c_dtype == 0:
        out = torch.full((M, ldc), float("nan"), device="cuda")
    else:
        out = torch.empty(M, ldc, device="cuda", dtype=torch.bfloat16)
    run_gemm(a_st, lda, a_mn, b_st, ldb, b_mn, out, ldc, c_dtype, M, N, K, alpha, beta)
    torch.cuda.synchronize()
    code = C.c_uint(0)
    _lib.call("glt_device_error", C.byref(code))
    assert code.value == 0
    return out[:, :N]


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", CASES)
def test_pair_gemm_f32_out(pair_mode, a_mn, b_mn, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 5 + N * 3 + K + a_mn * 2 + b_mn)
    a_log, a_st, lda = _operand(M, K, a_mn, g)
    b_log, b_st, ldb = _operand(N, K, b_mn, g)
    pair = _gemm(a_st, lda, a_mn, b_st, ldb, b_mn, M, N, K, True)
    ref = a_log @ b_log.t()
    torch.testing.assert_close(pair, ref, rtol=2e-3, atol=2e-3 * K ** 0.5)
    single = _gemm(a_st, lda, a_mn, b_st, ldb, b_mn, M, N, K, False)
    # same products in the same K order on the tensor cores
    torch.testing.assert_close(pair, single, rtol=1e-5, atol=1e-5 * K ** 0.5)


def test_pair_gemm_bf16_out(pair_mode):
    M, N, K = 512, 4096, 512
    g = torch.Generator(device="cuda").manual_seed(12)
    a_log, a_st, lda = _operand(M, K, 0, g)
    b_log, b_st, ldb = _operand(N, K, 1, g)
    out = _gemm(a_st, lda, 0, b_st, ldb, 1, M, N, K, True, c_dtype=1)
    ref = (a_log @ b_log.t()).to(torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)


def test_pair_gemm_alpha_beta(pair_mode):
    M, N, K = 640, 2304, 192
    g = torch.Generator(device="cuda").manual_seed(6)
    a_log, a_st, lda = _operand(M, K, 0, g)
    b_log, b_st, ldb = _operand(N, K, 0, g)
    base = torch.randn(M, N, generator=g, device="cuda")
    out = _gemm(a_st, lda, 0, b_st, ldb, 0, M, N, K, True, alpha=0.5, beta=1.0, base=base)
    ref = 0.5 * (a_log @ b_log.t()) + base
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-2)
