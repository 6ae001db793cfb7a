"""The six stand-alone graft GEMMs and the shadow bake on the GPU, through the
C ABI: the reference's golden vectors (tiny S=3/H=2 shapes that need the
workspace packing path), random shapes against the oracle's orientation
functions, and bit-exact bakes including the H=513 sentinel with masks and
the double-bake guard."""
import ctypes as C
import json
import os

import numpy as np
import pytest
import torch

from glt_b200 import _lib
from oracle import bitexact as bx
from oracle import graft_ops as go

pytestmark = pytest.mark.gpu
lib = _lib.lib
KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))
EXPAND_FWD, CONTRACT_FWD, EXPAND_WGRAD, CONTRACT_WGRAD, EXPAND_DGRAD, CONTRACT_DGRAD = range(6)


@pytest.fixture(scope="module")
def arena():
    a = C.c_void_p()
    _lib.check(lib.glt_arena_create(64 << 20, C.byref(a)))
    yield a
    lib.glt_arena_destroy(a)


def vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def op(code, M, S, H, w, x=None, dy=None, out=None, arena=None, alpha=1.0, beta=0.0, x_f32=False,
       dy_f32=False, w_bf16=None):
    s = torch.cuda.current_stream().cuda_stream
    xs = x.stride(0) if x is not None else 0
    ds = dy.stride(0) if dy is not None else 0
    _lib.check(lib.glt_graft_op(code, M, S, H, vp(w), vp(w_bf16), vp(x), int(x_f32), xs, vp(dy),
                                int(dy_f32), ds, vp(out), out.stride(0), alpha, beta, arena,
                                C.c_void_p(s)))
    torch.cuda.synchronize()
    return out


def cu(a, dtype=torch.float32):
    return torch.tensor(np.asarray(a), dtype=dtype, device="cuda")


def test_contract_audit_golden_vectors(arena):
    k = KATS["contract_audit"]
    S, H, M = k["S"], k["H"], k["M"]
    ex = k["expected"]
    W = cu(k["delta_exp"])                          # [S,H]
    Wc = cu(np.array(k["delta_ctr_tphs"]).T.copy())  # storage [S,H]
    x_h = cu(k["x_h"], torch.bfloat16)
    x_i = cu(k["x_i"], torch.bfloat16)
    dy_s = cu(k["dy_s"], torch.bfloat16)
    dx_h = cu(k["dx_h"], torch.bfloat16)
    o = op(EXPAND_FWD, M, S, H, W, x=x_h, out=torch.zeros(M, S, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu(), ex["expand_forward"], atol=1e-5)
    o = op(EXPAND_WGRAD, M, S, H, None, x=x_h, dy=dy_s, out=torch.zeros(S, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu(), ex["expand_weight_grad"], atol=1e-5)
    o = op(EXPAND_DGRAD, M, S, H, W, dy=dy_s, out=torch.zeros(M, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu(), ex["expand_input_grad"], atol=1e-5)
    o = op(CONTRACT_FWD, M, S, H, Wc, x=x_i, out=torch.zeros(M, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu(), ex["contract_forward"], atol=1e-5)
    o = op(CONTRACT_WGRAD, M, S, H, None, x=x_i, dy=dx_h, out=torch.zeros(S, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu().T, ex["contract_weight_grad_math_HS"], atol=1e-5)
    o = op(CONTRACT_DGRAD, M, S, H, Wc, dy=dx_h, out=torch.zeros(M, S, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu(), ex["contract_input_grad"], atol=1e-5)


def test_down_orientation_and_strided_input(arena):
    k = KATS["down_orientation"]
    S, H, M, F = k["S"], k["H"], k["M"], k["intermediate_stride"]
    W = cu(np.array(k["W_storage_SH_flat"]).reshape(S, H))
    x = torch.zeros(M, F, dtype=torch.bfloat16, device="cuda")
    x[:, :S] = cu(k["X"], torch.bfloat16)
    o = op(CONTRACT_FWD, M, S, H, W, x=x, out=torch.zeros(M, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu().reshape(-1), k["expected_forward"], atol=1e-5)
    dy = cu(k["dY"])
    o = op(CONTRACT_WGRAD, M, S, H, None, x=x, dy=dy, dy_f32=True, out=torch.zeros(S, H, device="cuda"), arena=arena)
    np.testing.assert_allclose(o.cpu().reshape(-1), k["expected_wgrad_storage_flat"], atol=1e-5)


def test_contract_probe(arena):
    k = KATS["contract_probe"]
    S, H, F, M = 32, 32, 64, k["M"]
    x = torch.zeros(M, F, dtype=torch.bfloat16, device="cuda")
    for r, c, v in k["inputs"]:
        x[r, c] = v
    W = torch.zeros(S, H, device="cuda")
    for s, h, v in k["weights"]:
        W[s, h] = v
    o = op(CONTRACT_FWD, M, S, H, W, x=x, out=torch.zeros(M, H, device="cuda"), arena=arena)
    exp = torch.zeros(M, H)
    for r, c, v in k["expected_nonzero"]:
        exp[r, c] = v
    torch.testing.assert_close(o.cpu(), exp, rtol=0, atol=1e-6)


@pytest.mark.parametrize("M,S,H", [(256, 128, 512), (300, 96, 136), (1024, 2752, 512)])
def test_random_shapes_vs_oracle(arena, M, S, H):
    g = torch.Generator().manual_seed(M + S + H)
    W = (torch.randn(S, H, generator=g) * 0.05)
    xh = torch.randn(M, H + 8, generator=g)[:, :H]        # strided view
    xi = torch.randn(M, S, generator=g)
    dys = torch.randn(M, S, generator=g)
    dyh = torch.randn(M, H, generator=g)
    Wd = W.cuda()
    bf = lambda t: t.contiguous().to(torch.bfloat16).cuda()
    xh_full = torch.randn(M, H + 8, generator=g)
    xh_full[:, :H] = xh
    xh_d = xh_full.to(torch.bfloat16).cuda()[:, :H]
    cases = [
        (EXPAND_FWD, dict(x=xh_d), go.expand_forward(xh.numpy(), W.numpy()), (M, S)),
        (CONTRACT_FWD, dict(x=bf(xi)), go.contract_forward(xi.numpy(), W.numpy()), (M, H)),
        (EXPAND_WGRAD, dict(x=xh_d, dy=dys.cuda(), dy_f32=True), go.expand_weight_grad(xh.numpy(), dys.numpy()), (S, H)),
        (CONTRACT_WGRAD, dict(x=bf(xi), dy=dyh.cuda(), dy_f32=True), go.contract_weight_grad(xi.numpy(), dyh.numpy()), (S, H)),
        (EXPAND_DGRAD, dict(dy=bf(dys)), go.expand_input_grad(dys.numpy(), W.numpy()), (M, H)),
        (CONTRACT_DGRAD, dict(dy=bf(dyh)), go.contract_input_grad(dyh.numpy(), W.numpy()), (M, S)),
    ]
    for code, kw, ref, shp in cases:
        w = None if code in (EXPAND_WGRAD, CONTRACT_WGRAD) else Wd
        o = op(code, M, S, H, w, out=torch.zeros(*shp, device="cuda"), arena=arena, **kw)
        torch.testing.assert_close(o.cpu(), torch.from_numpy(ref), rtol=2e-3, atol=2e-3 * (M ** 0.5))


def test_alpha_beta_accumulate_into_slice(arena):
    # ContractInputGrad accumulates (beta=1) into the i-slice of a wider fp32 buffer
    M, S, H, F, i0 = 64, 16, 32, 96, 32
    g = torch.Generator().manual_seed(9)
    W = torch.randn(S, H, generator=g).cuda()
    dy = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    gi = torch.randn(M, F, generator=g).cuda()
    base = gi.clone()
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.glt_graft_op(CONTRACT_DGRAD, M, S, H, vp(W), None, None, 0, 0, vp(dy), 0, H,
                                C.c_void_p(gi.data_ptr() + i0 * 4), F, 1.0, 1.0, arena, C.c_void_p(s)))
    torch.cuda.synchronize()
    ref = base.clone()
    ref[:, i0:i0 + S] += dy.float() @ W.to(torch.bfloat16).float().t()
    torch.testing.assert_close(gi, ref, rtol=1e-3, atol=1e-2)


def test_workspace_too_small_reports_need():
    a = C.c_void_p()
    _lib.check(lib.glt_arena_create(0, C.byref(a)))
    W = torch.zeros(3, 2, device="cuda")
    x = torch.zeros(2, 2, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(2, 3, device="cuda")
    st = lib.glt_graft_op(EXPAND_FWD, 2, 3, 2, vp(W), None, vp(x), 0, 2, None, 0, 0, vp(out), 3,
                          1.0, 0.0, a, None)
    lib.glt_arena_destroy(a)
    assert st == 7 and "workspace" in _lib.last_error()


def bake_gpu(base_bits: np.ndarray, graft: np.ndarray, i0, h0, mode):
    b = torch.from_numpy(base_bits.astype(np.int16)).cuda()
    g = torch.from_numpy(graft.astype(np.float32)).cuda()
    _lib.check(lib.glt_shadow_bake(vp(b), base_bits.shape[1], vp(g), graft.shape[0], graft.shape[1],
                                   i0, h0, mode, None))
    torch.cuda.synchronize()
    return b.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("mode", [0, 1])
def test_shadow_bake_bit_exact_random(mode):
    rng = np.random.default_rng(mode)
    S, H, i0, h0 = 37, 300, 11, 7
    rows, cols = (64, 320) if mode == 0 else (320, 64)
    base = bx.f32_to_bf16_bits(rng.standard_normal((rows, cols)).astype(np.float32))
    g = (rng.standard_normal((S, H)) * 0.01).astype(np.float32)
    got = bake_gpu(base, g, i0, h0, mode)
    ref = base.copy()
    bx.shadow_bake_kernel(ref, g, i0, h0, mode)
    np.testing.assert_array_equal(got, ref)


def test_apply_graft_to_shadow_h513_sentinel_masks_guard():
    from glt_b200 import graft as G
    k = KATS["bake_sentinel_h513"]
    S, H, L = k["S"], k["H"], k["num_layers"]
    flat = np.zeros(L * 3 * S * H, np.float32)
    for l in range(L):
        for p in range(3):
            s = np.arange(S)[:, None]
            h = np.arange(H)[None, :]
            off = bx.delta_offset(l, p, S, H)
            flat[off:off + S * H] = ((l * 100 + p * 10 + s) * 1000 + h + 1).ravel()

    def run(gate, up, down, start, end, twice=False):
        cfg = G.default_config()
        cfg.num_layers, cfg.slice_dim, cfg.hidden_dim, cfg.intermediate_dim = L, S, H, S
        cfg.max_domains, cfg.domain_id = 1, 0
        cfg.graft_proj_gate, cfg.graft_proj_up, cfg.graft_proj_down = gate, up, down
        cfg.graft_layer_start, cfg.graft_layer_end = start, end
        ws = [[torch.zeros(S, H, dtype=torch.int16, device="cuda") for _ in range(L)] for _ in range(2)]
        wd = [torch.zeros(H, S, dtype=torch.int16, device="cuda") for _ in range(L)]
        arr = lambda ts: (C.c_void_p * L)(*[t.data_ptr() for t in ts])
        g = torch.from_numpy(flat).cuda()
        flag = C.c_int(0)
        st = lib.glt_apply_graft_to_shadow(C.byref(cfg.to_c()), arr(ws[0]), arr(ws[1]), arr(wd), H, S,
                                           vp(g), C.byref(flag), None)
        assert st == 0, _lib.last_error()
        if twice:
            st2 = lib.glt_apply_graft_to_shadow(C.byref(cfg.to_c()), arr(ws[0]), arr(ws[1]), arr(wd),
                                                H, S, vp(g), C.byref(flag), None)
            assert st2 == 6
        # oracle
        layers = [dict(gate=np.zeros((S, H), np.uint16), up=np.zeros((S, H), np.uint16),
                       down=np.zeros((H, S), np.uint16)) for _ in range(L)]

        class Cfg:
            num_layers, slice_dim, h_slice_dim = L, S, H
            graft_layer_start, graft_layer_end = start, end
            graft_proj_gate, graft_proj_up, graft_proj_down = gate, up, down
        bx.apply_graft_to_shadow(layers, flat, Cfg, bx.ShadowBakeState(), 0)
        for l in range(L):
            for name, t in (("gate", ws[0][l]), ("up", ws[1][l]), ("down", wd[l])):
                np.testing.assert_array_equal(t.cpu().numpy().view(np.uint16), layers[l][name])

    run(1, 1, 1, 0, L - 1, twice=True)
    run(0, 0, 1, 0, L - 1)
    run(1, 1, 1, 1, 1)
