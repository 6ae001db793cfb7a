"""Stand-alone layer kernels through the C ABI against the fp32 oracle:
glt_rmsnorm_fwd / glt_rmsnorm_bwd (rms_norm_fwd_kernel / rms_norm_bwd_kernel,
src/kernels_rmsnorm_kernels.inc:8-126; the backward with and without the
residual) and glt_rope (apply_rope, src/rope_impl.inc:8-64: half-split
rotation of the q and k heads in place, v untouched, and its transpose)."""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib
from oracle import ref_math as rm
from tests.parity import assert_close_bf16, bf16r

pytestmark = pytest.mark.gpu
lib = _lib.lib


def vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,D", [(300, 896), (64, 4096), (1, 256)])
def test_rmsnorm_forward_and_backward(M, D):
    g = torch.Generator().manual_seed(M + D)
    x = bf16r(torch.randn(M, D, generator=g) * 2)
    w = bf16r(1 + 0.1 * torch.randn(D, generator=g))
    eps = 1e-6
    xd, wd = x.to("cuda", torch.bfloat16), w.to("cuda", torch.bfloat16)
    y = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")
    var = torch.empty(M, device="cuda")
    _lib.check(lib.glt_rmsnorm_fwd(vp(xd), vp(wd), vp(y), vp(var), M, D, eps, stream()))
    torch.cuda.synchronize()
    y_ref, var_ref = rm.rms_norm(x, w, eps)
    assert_close_bf16(y.float().cpu(), y_ref, "rmsnorm y")
    torch.testing.assert_close(var.cpu(), var_ref, rtol=1e-5, atol=1e-7)

    dy = torch.randn(M, D, generator=g)
    resid = torch.randn(M, D, generator=g)
    dx_ref = rm.rms_norm_bwd(dy, x, w, var_ref, eps)
    dyd, rd = dy.cuda(), resid.cuda()
    for with_resid in (False, True):
        dx = torch.empty(M, D, device="cuda")
        _lib.check(lib.glt_rmsnorm_bwd(vp(dyd), vp(xd), vp(wd), vp(var), vp(rd) if with_resid else None,
                                       vp(dx), M, D, eps, stream()))
        torch.cuda.synchronize()
        want = dx_ref + resid if with_resid else dx_ref
        torch.testing.assert_close(dx.cpu(), want, rtol=2e-4, atol=2e-5)


@pytest.mark.parametrize("B,T,nh,nkv,hd,theta", [(2, 128, 4, 2, 64, 10000.0), (1, 256, 8, 2, 128, 500000.0),
                                                 (2, 64, 14, 2, 64, 1000000.0)])
def test_rope_forward_and_inverse(B, T, nh, nkv, hd, theta):
    g = torch.Generator().manual_seed(T + nh)
    QKV = (nh + 2 * nkv) * hd
    qkv = bf16r(torch.randn(B * T, QKV, generator=g))
    d = qkv.to("cuda", torch.bfloat16)
    _lib.check(lib.glt_rope(vp(d), QKV, B, T, nh, nkv, hd, theta, 0, stream()))
    torch.cuda.synchronize()
    cos, sin = rm.rope_tables(T, hd, theta)
    q = rm.apply_rope(qkv[:, :nh * hd].view(B, T, -1), nh, hd, cos, sin).reshape(B * T, -1)
    k = rm.apply_rope(qkv[:, nh * hd:(nh + nkv) * hd].view(B, T, -1), nkv, hd, cos, sin).reshape(B * T, -1)
    got = d.float().cpu()
    assert_close_bf16(got[:, :nh * hd], q, "rope q")
    assert_close_bf16(got[:, nh * hd:(nh + nkv) * hd], k, "rope k")
    assert torch.equal(got[:, (nh + nkv) * hd:], qkv[:, (nh + nkv) * hd:])       # v untouched
    # the inverse (the backward's transpose rotation) brings q and k back
    _lib.check(lib.glt_rope(vp(d), QKV, B, T, nh, nkv, hd, theta, 1, stream()))
    torch.cuda.synchronize()
    assert_close_bf16(d.float().cpu(), qkv, "rope inverse round trip")


def test_rope_table_cache_is_bounded_and_still_correct():
    # more (seq_len, theta) pairs than the cache holds: evicted tables are
    # rebuilt and the results stay right
    nh, nkv, hd, B = 2, 1, 64, 1
    QKV = (nh + 2 * nkv) * hd
    for i in range(12):
        T = 64 * (1 + i % 6)
        theta = 10000.0 * (1 + i // 6)
        g = torch.Generator().manual_seed(i)
        qkv = bf16r(torch.randn(B * T, QKV, generator=g))
        d = qkv.to("cuda", torch.bfloat16)
        _lib.check(lib.glt_rope(vp(d), QKV, B, T, nh, nkv, hd, theta, 0, stream()))
        torch.cuda.synchronize()
        cos, sin = rm.rope_tables(T, hd, theta)
        q = rm.apply_rope(qkv[:, :nh * hd].view(B, T, -1), nh, hd, cos, sin).reshape(B * T, -1)
        assert_close_bf16(d.float().cpu()[:, :nh * hd], q, f"rope q (T {T}, theta {theta})")
