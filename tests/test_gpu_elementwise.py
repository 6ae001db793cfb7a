"""Stand-alone bandwidth-bound ops through the C ABI against the fp32 oracle:
glt_swiglu_fwd / glt_swiglu_bwd (fused_silu_product_strided_kernel and
fused_gate_up_bwd_kernel, kernels_elementwise_impl.inc:80-124,411-448),
glt_adamw_all (execute_adamw_all, kernels_optimizer_impl.inc:11-77), and the
fused bf16 weight image the model's AdamW refreshes after each step."""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib
from glt_b200 import graft as G
from oracle import bitexact as bx
from oracle import ref_math as rm
from tests.parity import to_glt_config

pytestmark = pytest.mark.gpu
lib = _lib.lib


def vp(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("rows,width,ld", [(3, 8, 8), (64, 688, 704), (257, 1024, 2048)])
def test_swiglu_fwd_strided_matches_oracle(rows, width, ld):
    g = torch.Generator(device="cuda").manual_seed(rows + width)
    gate = (torch.randn(rows, ld, device="cuda", generator=g) * 3).to(torch.bfloat16)
    up = torch.randn(rows, ld + 8, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.full((rows, ld + 16), 7.0, device="cuda", dtype=torch.bfloat16)
    _lib.check(lib.glt_swiglu_fwd(vp(gate), vp(up), vp(out), rows, width, ld, ld + 8, ld + 16, stream()))
    torch.cuda.synchronize()
    ref = rm.silu_product(gate[:, :width].cpu(), up[:, :width].cpu())
    got = out[:, :width].cpu()
    # bf16 outputs from fp32 math: identical up to one bf16 ulp where exp differs in its last bit
    diff = (got.float() - ref.float()).abs()
    ulp = ref.float().abs().clamp_min(1e-30) * 2.0 ** -7
    assert bool((diff <= ulp).all())
    assert float((got != ref).float().mean()) < 1e-3
    assert bool((out[:, width:] == 7.0).all()), "wrote outside the row width"


def test_swiglu_bwd_matches_oracle():
    n = 3 * 4096 + 8
    g = torch.Generator(device="cuda").manual_seed(5)
    gate = (torch.randn(n, device="cuda", generator=g) * 3).to(torch.bfloat16)
    up = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    gi = torch.randn(n, device="cuda", generator=g)
    dg = torch.empty(n, device="cuda")
    du = torch.empty(n, device="cuda")
    _lib.check(lib.glt_swiglu_bwd(vp(dg), vp(du), vp(gi), vp(up), vp(gate), n, stream()))
    torch.cuda.synchronize()
    rg, ru = rm.gate_up_backward(gi.cpu(), up.cpu(), gate.cpu())
    torch.testing.assert_close(dg.cpu(), rg, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(du.cpu(), ru, rtol=1e-5, atol=1e-6)


def test_swiglu_rejects_bad_shapes():
    t = torch.zeros(64, device="cuda", dtype=torch.bfloat16)
    assert lib.glt_swiglu_fwd(vp(t), vp(t), vp(t), 1, 12, 16, 16, 16, stream()) == 1
    assert "multiples of 8" in _lib.last_error()
    f = torch.zeros(64, device="cuda")
    assert lib.glt_swiglu_bwd(vp(f), vp(f), vp(f), vp(t), vp(t), 12, stream()) == 1
    assert lib.glt_swiglu_fwd(vp(t), vp(t), vp(t), 0, 8, 8, 8, 8, stream()) == 0   # empty: no-op


@pytest.mark.parametrize("projs", [(1, 1, 1), (0, 0, 1)])
@pytest.mark.parametrize("with_scale", [False, True])
def test_adamw_all_matches_oracle(projs, with_scale):
    rc = rm.GraftConfig(hidden_dim=256, intermediate_dim=640, slice_dim=64, num_layers=3,
                        graft_proj_gate=projs[0], graft_proj_up=projs[1], graft_proj_down=projs[2],
                        layout="concat", adam_weight_decay=0.01).finalize()
    n = rc.total_projections * rc.slice_dim * rc.h_slice_dim
    g = torch.Generator().manual_seed(9)
    w = torch.randn(n, generator=g) * 0.02
    grad = torch.randn(n, generator=g) * 1e-3
    m = torch.randn(n, generator=g) * 1e-4
    v = torch.rand(n, generator=g) * 1e-6
    scale = 0.37 if with_scale else 1.0
    dw, dg, dm, dv = (t.cuda() for t in (w, grad, m, v))
    img = torch.zeros(n, dtype=torch.int16, device="cuda")
    ds = torch.tensor([scale], device="cuda") if with_scale else None
    cfg = to_glt_config(rc).to_c()
    step, lr = 4, 3e-4
    _lib.check(lib.glt_adamw_all(vp(dw), vp(img), vp(dg), vp(dm), vp(dv), vp(ds), C.byref(cfg), step,
                                 lr, stream()))
    torch.cuda.synchronize()
    rw, rmm, rvv = w.clone(), m.clone(), v.clone()
    rm.adamw(rw, grad * scale, rmm, rvv, step, lr, rc)
    torch.testing.assert_close(dw.cpu(), rw, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(dm.cpu(), rmm, rtol=1e-6, atol=1e-9)
    torch.testing.assert_close(dv.cpu(), rvv, rtol=1e-6, atol=1e-12)
    # bf16 image: RNE of the updated weight where the projection is enabled, untouched elsewhere
    want = torch.from_numpy(bx.f32_to_bf16_bits(dw.cpu().numpy()).astype("int16"))
    SH = rc.slice_dim * rc.h_slice_dim
    for proj in range(rc.total_projections):
        sl = slice(proj * SH, (proj + 1) * SH)
        if projs[proj % 3]:
            assert torch.equal(img.cpu()[sl], want[sl])
        else:
            assert bool((img.cpu()[sl] == 0).all())


def test_fused_weight_image_tracks_master_after_steps():
    """After AdamW, the bf16 graft columns inside the fused [base | graft]
    weights equal RNE(bf16) of the fp32 master: gate/up rows (128-row
    interleave) and the transposed down columns."""
    rc = rm.GraftConfig(hidden_dim=256, intermediate_dim=640, slice_dim=192, vocab_size=512,
                        num_layers=3, num_heads=4, num_kv_heads=2, graft_layer_start=1,
                        graft_layer_end=2, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                        layout="concat", lr_peak=1e-2,
                        lr_warmup_steps=1).finalize()
    B, T = 2, 128
    m = G.GraftModel(to_glt_config(rc), B, T, kind=G.MODEL_DECODER)
    m.init_random(seed=3, std=0.02, graft_std=0.02, graft_down_std=0.02)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=g, dtype=torch.int32)
    ood = torch.zeros(B, T, dtype=torch.int32)
    ood[1:] = 1
    for step in range(2):
        m.train_step(ids, ood, step, 4)
    torch.cuda.synchronize()
    master = m.read_graft("weight").cpu().view(rc.num_layers, 3, rc.slice_dim, rc.h_slice_dim)
    bits = lambda t: torch.from_numpy(bx.f32_to_bf16_bits(t.numpy()).astype("int16"))
    D, F, S = rc.hidden_dim, rc.intermediate_dim, rc.slice_dim
    F_pad = (F + 255) // 256 * 256
    FF = F_pad + (S + 127) // 128 * 128
    c = F_pad + torch.arange(S)
    gate_rows = 256 * (c // 128) + c % 128
    for l in range(rc.num_layers):
        wgu = m.activation(7, l).view(torch.int16).cpu().view(2 * FF, D)
        wd = m.activation(8, l).view(torch.int16).cpu().view(D, FF)
        if l < rc.graft_layer_start:   # ungrafted layer: its graft columns stay zero
            assert bool((wgu[gate_rows] == 0).all()) and bool((wd[:, F_pad:F_pad + S] == 0).all())
            continue
        assert torch.equal(wgu[gate_rows], bits(master[l, 0])), f"gate image L{l}"
        assert torch.equal(wgu[gate_rows + 128], bits(master[l, 1])), f"up image L{l}"
        assert torch.equal(wd[:, F_pad:F_pad + S], bits(master[l, 2]).t()), f"down image L{l}"
    m.close()


@pytest.mark.parametrize("n,gscale,apply", [(4096 * 3 + 5, 1e-2, 1), (1 << 20, 1e-5, 1), (777, 1.0, 0)])
def test_grad_clip_matches_oracle(n, gscale, apply):
    g = torch.randn(n, generator=torch.Generator().manual_seed(n)) * gscale
    dg = g.cuda()
    work = torch.empty(1024, dtype=torch.float64, device="cuda")
    scale = torch.empty(1, device="cuda")
    norm = torch.empty(1, device="cuda")
    _lib.check(lib.glt_grad_clip(vp(dg), n, 1.0, apply, vp(work), work.numel() * 8, vp(scale), vp(norm),
                                 stream()))
    torch.cuda.synchronize()
    ref = g.clone()
    ref_norm, ref_scale = rm.clip_grads(ref, 1.0)
    assert float(norm) == pytest.approx(ref_norm, rel=1e-5)
    assert float(scale) == pytest.approx(ref_scale, rel=1e-5)
    torch.testing.assert_close(dg.cpu(), ref if apply else g, rtol=1e-6, atol=0)


def test_grad_clip_rejects_small_workspace():
    dg = torch.zeros(64, device="cuda")
    work = torch.empty(16, dtype=torch.float64, device="cuda")
    scale = torch.empty(1, device="cuda")
    assert lib.glt_grad_clip(vp(dg), 64, 1.0, 1, vp(work), 128, vp(scale), None, stream()) == 1
    assert "workspace" in _lib.last_error()
