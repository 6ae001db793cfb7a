"""Failure detection on the GPU without a GPU fault.

Every tcgen05 kernel bounds its mbarrier waits.  glt_selftest_wait_timeout
runs a small GEMM in which one CTA never receives its first k-block (a
barrier that nothing completes), with a 20 ms bound instead of the usual 4 s:
that CTA gives up, records the code in the device error word, drains its
copies and tensor-core work and exits.  The checks: the timeout reaches the
caller as GLT_ETIMEOUT (the reference throws from its CHECK macros,
src/checks.hpp:10-44), a model call reports a code left pending by an
earlier kernel and then runs clean, and the next launches on the device are
unaffected (the error word is not consulted by later launches)."""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib

pytestmark = pytest.mark.gpu
lib = _lib.lib
ETIMEOUT = 5


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def device_error():
    v = C.c_uint()
    _lib.check(lib.glt_device_error(C.byref(v)))
    return v.value


def gemm_ok(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(384, 512, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(640, 512, device="cuda", generator=g).to(torch.bfloat16)
    c = torch.empty(384, 640, device="cuda")
    _lib.check(lib.glt_gemm(C.c_void_p(a.data_ptr()), 512, 0, C.c_void_p(b.data_ptr()), 512, 0,
                            C.c_void_p(c.data_ptr()), 640, 0, 384, 640, 512, 1.0, 0.0, stream()))
    torch.cuda.synchronize()
    torch.testing.assert_close(c, a.float() @ b.float().t(), rtol=1e-3, atol=1e-3)


def test_wait_timeout_is_reported_and_the_next_launch_is_clean():
    assert device_error() == 0
    st = lib.glt_selftest_wait_timeout(20, 0, stream())
    assert st == ETIMEOUT, _lib.last_error()
    assert "bounded device wait" in _lib.last_error()
    assert device_error() == 0          # read and cleared by the call
    for seed in range(3):               # later launches wait their full bound and finish
        gemm_ok(seed)
    assert device_error() == 0


def test_pending_timeout_is_reported_by_the_next_model_step():
    from tests.test_gpu_decoder import gpu_model, problem, small_cfg
    rc = small_cfg()
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T)
    try:
        assert lib.glt_selftest_wait_timeout(20, 1, stream()) == 0
        # enqueued without stats: the step itself cannot report it ...
        m.train_step(ids, ood, 0, 4, want_stats=False)
        # ... its stats do
        with pytest.raises(_lib.GltError) as e:
            m.step_stats(0)
        assert e.value.status == ETIMEOUT
        st = m.train_step(ids, ood, 1, 4)   # clean again
        assert st["total_loss"] > 0
        # a forward collects a pending code for the model's next read-back
        assert lib.glt_selftest_wait_timeout(20, 1, stream()) == 0
        m.forward(ids.cuda(), want_logits=False)
        with pytest.raises(_lib.GltError) as e:
            m.train_step(ids, ood, 2, 4)
        assert e.value.status == ETIMEOUT
        m.train_step(ids, ood, 3, 4)
    finally:
        m.close()
    assert device_error() == 0
