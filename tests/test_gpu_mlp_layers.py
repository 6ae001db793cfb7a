"""Layer-level grafted MLP through the C ABI (glt_mlp_*) and stand-alone graft
weights (glt_graft_weights_alloc / _free), against the fp32 oracle.

A caller that keeps the reference's own layer loop replaces the MLP half of
forward_layer (src/layer_forward_impl.inc:53-285), recompute_ffn
(src/layer_recompute_impl.inc:8-91) and the MLP half of backward_layer with
the post-attention RMSNorm backward (src/layer_backward_impl.inc:36-367)
call for call.  For each layer of a two-layer stack, in both graft
geometries: the forward output and the saved tensors, then the backward's
input gradient and the layer's graft gradients, with the gate_pre/up store
from glt_mlp_recompute and with the recompute fused into the backward GEMM.
"""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib
from oracle import ref_math as rm
from tests.parity import assert_close_bf16, bf16r, make_decoder_weights, to_glt_config

pytestmark = pytest.mark.gpu
lib = _lib.lib
W_POST_NORM, W_GATE, W_UP, W_DOWN = 8, 9, 10, 11


def vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def cfg(layout):
    kw = dict(hidden_dim=256, intermediate_dim=640, num_layers=2, num_heads=4, num_kv_heads=4,
              vocab_size=64, graft_layer_start=0, graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1,
              graft_proj_down=1, lambda_silence=5.0, layout=layout)
    if layout == "concat":
        kw.update(slice_dim=128)
    else:                                   # slice [40, 80) x hidden [64, 128): off the tile grids
        kw.update(slice_dim=40, max_domains=4, domain_id=1)
    return rm.GraftConfig(**kw).finalize()


@pytest.mark.parametrize("layout", ["concat", "overlay"])
def test_layer_calls_match_oracle(layout):
    rc = cfg(layout)
    M, D, S, H = 256, rc.hidden_dim, rc.slice_dim, rc.h_slice_dim
    w = make_decoder_weights(rc, seed=5, std=0.05)
    g = torch.Generator().manual_seed(6)
    delta = torch.randn(rc.total_projections * S * H, generator=g) * 0.05
    x_post = bf16r(torch.randn(M, D, generator=g))
    dy = torch.randn(M, D, generator=g) * 0.1
    ood = (torch.rand(M, generator=g) < 0.4).to(torch.int32)
    ood_d = ood.cuda()
    lam = 3e-3
    c = to_glt_config(rc).to_c()

    gw = _lib.GltGraftWeights()
    _lib.check(lib.glt_graft_weights_alloc(C.byref(c), rc.domain_id, 1, C.byref(gw)))
    mlp = C.c_void_p()
    _lib.check(lib.glt_mlp_create(C.byref(c), M, C.byref(mlp)))
    try:
        assert gw.allocated == 1 and gw.active == 0 and gw.weight_elems == delta.numel()
        zero = torch.empty(delta.numel(), device="cuda")
        _lib.call("glt_memcpy", vp(zero), C.c_void_p(gw.weight), delta.numel() * 4, stream(), 1)
        assert float(zero.abs().max()) == 0.0                            # zero-initialised
        for l, lw in enumerate(w["layers"]):
            for which, t in ((W_POST_NORM, lw["post_norm"]), (W_GATE, lw["wg"]), (W_UP, lw["wu"]),
                             (W_DOWN, lw["wd"])):
                tb = t.to(device="cuda", dtype=torch.bfloat16).contiguous()
                _lib.check(lib.glt_mlp_set_weight(mlp, l, which, vp(tb), tb.numel(), 0, stream()))
        dl = delta.cuda()
        _lib.call("glt_memcpy", C.c_void_p(gw.weight), vp(dl), dl.numel() * 4, stream(), 1)
        gw.active = 1
        _lib.check(lib.glt_mlp_set_graft(mlp, C.byref(gw), stream()))
        mirror = torch.empty(delta.numel(), dtype=torch.bfloat16, device="cuda")
        _lib.call("glt_memcpy", vp(mirror), C.c_void_p(gw.weight_bf16), delta.numel() * 2, stream(), 1)
        assert torch.equal(mirror.cpu(), delta.to(torch.bfloat16))      # bf16 mirror, RNE
        nbytes = C.c_int64()
        _lib.check(lib.glt_mlp_recompute_bytes(mlp, C.byref(nbytes)))
        gate_up = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")

        xp = x_post.to(device="cuda", dtype=torch.bfloat16)
        for l in range(rc.num_layers):
            lw = w["layers"][l]
            x_ffn = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")
            var = torch.empty(M, device="cuda")
            esq = torch.empty(3, M, device="cuda")
            dd = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
            saved = _lib.GltMlpSaved(x_ffn.data_ptr(), var.data_ptr(), esq.data_ptr(), dd.data_ptr())
            x_out = torch.empty_like(xp)
            _lib.check(lib.glt_mlp_fwd(mlp, l, vp(xp), vp(x_out), C.byref(saved), 1, stream()))
            torch.cuda.synchronize()

            xn, var_ref = rm.rms_norm(x_post, lw["post_norm"], rc.rms_norm_eps)
            ffn, sv = rm.mlp_forward(xn, lw, delta, rc, l)
            what = f"{layout} L{l}"
            assert_close_bf16(x_out.float().cpu(), x_post + ffn, f"{what} x_out")
            assert_close_bf16(x_ffn.float().cpu(), xn, f"{what} x_ffn")
            torch.testing.assert_close(var.cpu(), var_ref, rtol=1e-4, atol=1e-6)
            for p, key, width in ((0, "energy_gate", S), (1, "energy_up", S), (2, "energy_down", H)):
                e_gpu = torch.sqrt(esq[p].cpu() + 1e-8) / width ** 0.5
                assert_close_bf16(e_gpu, sv[key], f"{what} {key}")
            assert_close_bf16(dd.float().cpu(), sv["delta_down"], f"{what} delta_down")

            g_ref = torch.zeros_like(delta)
            dffn = rm.mlp_backward(dy, xn, lw, delta, sv, rc, l, ood, lam, g_ref)
            dx_ref = dy + rm.rms_norm_bwd(dffn, x_post, lw["post_norm"], var_ref, rc.rms_norm_eps)
            SH = S * H
            for mode in ("store", "fused"):
                dx = dy.cuda().contiguous()
                grad = torch.full((delta.numel(),), 7.0, device="cuda")   # stale values get overwritten
                gu = None
                if mode == "store":
                    _lib.check(lib.glt_mlp_recompute(mlp, l, C.byref(saved), vp(gate_up), stream()))
                    gu = gate_up
                _lib.check(lib.glt_mlp_bwd(mlp, l, vp(dx), vp(xp), C.byref(saved), vp(gu), vp(ood_d),
                                           lam, vp(grad), stream()))
                torch.cuda.synchronize()
                assert_close_bf16(dx.cpu(), dx_ref, f"{what} {mode} dx")
                gg = grad.cpu()
                for p, name in enumerate(("gate", "up", "down")):
                    sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
                    assert_close_bf16(gg[sl], g_ref[sl], f"{what} {mode} grad {name}")
                other = torch.ones_like(gg, dtype=torch.bool)
                other[3 * l * SH:3 * (l + 1) * SH] = False
                assert bool((gg[other] == 7.0).all())                     # other layers untouched
        err = C.c_uint()
        _lib.check(lib.glt_device_error(C.byref(err)))
        assert err.value == 0
    finally:
        lib.glt_mlp_destroy(mlp)
        _lib.check(lib.glt_graft_weights_free(C.byref(gw)))
    assert (gw.weight, gw.weight_bf16, gw.weight_elems, gw.allocated, gw.active) == (None, None, 0, 0, 0)
    _lib.check(lib.glt_graft_weights_free(C.byref(gw)))                  # freeing twice is safe


def test_graft_weights_without_mirror_and_refusals():
    rc = cfg("overlay")
    c = to_glt_config(rc).to_c()
    gw = _lib.GltGraftWeights()
    _lib.check(lib.glt_graft_weights_alloc(C.byref(c), 2, 0, C.byref(gw)))
    try:
        assert gw.weight_bf16 is None and gw.domain_id == 2
        assert gw.weight_elems == 3 * rc.num_layers * rc.slice_dim * (rc.hidden_dim // rc.max_domains)
        # re-allocation frees the previous buffers first
        _lib.check(lib.glt_graft_weights_alloc(C.byref(c), 1, 1, C.byref(gw)))
        assert gw.weight_bf16 is not None and gw.domain_id == 1
        mlp = C.c_void_p()
        c2 = to_glt_config(cfg("concat")).to_c()
        _lib.check(lib.glt_mlp_create(C.byref(c2), 128, C.byref(mlp)))
        try:
            assert lib.glt_mlp_set_graft(mlp, C.byref(gw), stream()) == 1        # wrong geometry
            assert "elements" in _lib.last_error()
            t = torch.zeros(10, dtype=torch.bfloat16, device="cuda")
            assert lib.glt_mlp_set_weight(mlp, 0, 4, vp(t), 10, 0, stream()) == 1  # attention weight
            assert lib.glt_mlp_set_weight(mlp, 2, W_GATE, vp(t), 10, 0, stream()) == 1  # no layer 2
        finally:
            lib.glt_mlp_destroy(mlp)
    finally:
        _lib.check(lib.glt_graft_weights_free(C.byref(gw)))
