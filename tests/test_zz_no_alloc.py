"""glt_graft_op_noalloc: the allocation-free graft op for callers that cannot
call cudaMalloc (a framework's caching allocator owns the device memory, or
a latency-critical path cannot take cudaMalloc's device synchronisation).

Through the C ABI, each op is run twice in a row with different inputs and
compared with glt_graft_op (which stages in a caller-allocated GltArena):
the same kernel on the same operands, so the results agree within the
graft-op tolerance of tests/test_gpu_graft_ops.py.  Also checks that a
request beyond the fixed 16 MiB workspace is refused with a clear error,
that repeated calls leave the device memory in use unchanged (the property
the entry point exists for), and that a timeout recorded in its own error
word is reported once by glt_device_error and then cleared.
This file needs no fixture from other test files; it runs alone or last."""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib

pytestmark = pytest.mark.gpu
lib = _lib.lib
OPS = range(6)  # GLT_GRAFT_EXPAND_FWD .. GLT_GRAFT_CONTRACT_DGRAD


def vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def operands(code, M, S, H, seed):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(S, H, generator=g) * 0.1).cuda()
    x_cols = H if code in (0, 2) else S
    dy_cols = S if code in (2, 4) else H
    x = torch.randn(M, x_cols + 5, generator=g).to(torch.bfloat16).cuda()[:, :x_cols]  # strided
    dy = torch.randn(M, dy_cols, generator=g).cuda()                                    # fp32
    out_shape = {0: (M, S), 1: (M, H), 2: (S, H), 3: (S, H), 4: (M, H), 5: (M, S)}[code]
    base = torch.randn(*out_shape, generator=g).cuda()
    return W, x, dy, base


def call(fn, code, M, S, H, W, x, dy, out, arena=None):
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [code, M, S, H, vp(W), None, vp(x), 0, x.stride(0), vp(dy), 1, dy.stride(0), vp(out),
            out.stride(0), 0.5, 1.0]
    if fn == "arena":
        return lib.glt_graft_op(*args, arena, s)
    return lib.glt_graft_op_noalloc(*args, s)


@pytest.mark.parametrize("code", OPS)
@pytest.mark.parametrize("M,S,H", [(2, 3, 2), (257, 96, 136)])
def test_noalloc_matches_arena_op_twice(code, M, S, H):
    arena = C.c_void_p()
    _lib.check(lib.glt_arena_create(32 << 20, C.byref(arena)))
    try:
        for rep in range(2):  # two calls in a row, different inputs
            W, x, dy, base = operands(code, M, S, H, seed=100 * rep + code)
            ref = base.clone()
            got = base.clone()
            _lib.check(call("arena", code, M, S, H, W, x, dy, ref, arena))
            _lib.check(call("noalloc", code, M, S, H, W, x, dy, got))
            torch.cuda.synchronize()
            torch.testing.assert_close(got, ref, rtol=2e-3, atol=2e-3 * (max(M, S) ** 0.5))
    finally:
        lib.glt_arena_destroy(arena)


def test_noalloc_rejects_oversize_workspace():
    S = H = 4096                      # fp32 weight staged as bf16: 32 MiB > 16 MiB
    W = torch.zeros(S, H, device="cuda")
    x = torch.zeros(8, H, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, S, device="cuda")
    st = lib.glt_graft_op_noalloc(0, 8, S, H, vp(W), None, vp(x), 0, H, None, 0, 0, vp(out), S,
                                  1.0, 0.0, None)
    assert st == 1
    assert "16777216-byte workspace" in _lib.last_error()


def used_bytes():
    used = C.c_int64()
    _lib.check(lib.glt_device_memory(C.byref(used), None))
    return used.value


def test_noalloc_calls_leave_device_memory_unchanged():
    M, S, H = 513, 256, 1024        # fp32 weight and fp32 dy: both staged in the workspace
    cases = [operands(code, M, S, H, seed=7 + code) for code in OPS]
    outs = [base.clone() for (_, _, _, base) in cases]
    for code in OPS:   # first calls: symbol lookup and lazy loading of each kernel variant
        _lib.check(call("noalloc", code, M, S, H, *cases[code][:3], outs[code]))
    torch.cuda.synchronize()
    before = used_bytes()
    for rep in range(3):
        for code in OPS:
            W, x, dy, _ = cases[code]
            _lib.check(call("noalloc", code, M, S, H, W, x, dy, outs[code]))
    torch.cuda.synchronize()
    assert used_bytes() == before


def test_noalloc_error_word_is_reported_then_cleared():
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    v = C.c_uint()
    _lib.check(lib.glt_device_error(C.byref(v)))
    assert v.value == 0
    # a GEMM that times out against this entry point's own word (mode 2)
    _lib.check(lib.glt_selftest_wait_timeout(20, 2, s))
    _lib.check(lib.glt_device_error(C.byref(v)))
    assert v.value == 1
    _lib.check(lib.glt_device_error(C.byref(v)))
    assert v.value == 0
    # the word is not sticky: the next calls wait their full bound and agree
    test_noalloc_matches_arena_op_twice(1, 257, 96, 136)
