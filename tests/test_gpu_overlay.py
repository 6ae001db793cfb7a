"""The reference's own overlay geometry in the fused training path: the graft
overlays intermediate columns [i0, i0+S) and hidden columns [h0, h0+H) of the
base MLP, i0 = domain_id*S, h0 = domain_id*H, H = hidden/max_domains
(layer_forward_impl.inc:21-22).  Forward activations, logits, losses, graft
gradients and the AdamW update against the fp32 oracle; the shadow bake of the
fused weights against the oracle's bit-exact bake; explicit vs baked eval
within the certify bake budget (deploy/config.sh:40, EPS_CE_BAKE = 0.02)."""
import numpy as np
import pytest
import torch

from oracle import bitexact as bx
from oracle import ref_math as rm
from tests.parity import assert_close_bf16, load_weights, make_decoder_weights, to_glt_config

pytestmark = pytest.mark.gpu


def ov_cfg(**over):
    # S = F/4 = 160 and i0 = 160 do not fall on the 128-column tile grid
    kw = dict(hidden_dim=256, intermediate_dim=640, slice_dim=160, max_domains=4, domain_id=1,
              vocab_size=512, num_layers=2, num_heads=4, num_kv_heads=2, rope_theta=10000.0,
              graft_layer_start=0, graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1,
              graft_proj_down=1, layout="overlay", lambda_silence=5.0, tie_embeddings=True)
    kw.update(over)
    return rm.GraftConfig(**kw).finalize()


def problem(rc, B, T, seed=0, std=0.05, graft_std=0.05):
    w = make_decoder_weights(rc, seed, std)
    g = torch.Generator().manual_seed(seed + 100)
    delta = torch.randn(rc.total_projections * rc.slice_dim * rc.h_slice_dim, generator=g) * graft_std
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=g, dtype=torch.int32)
    ood = torch.zeros(B, T, dtype=torch.int32)
    ood[B // 2:] = 1
    return w, delta, ids, ood


def gpu_model(rc, w, delta, B, T):
    from glt_b200 import graft as G
    m = G.GraftModel(to_glt_config(rc), B, T, kind=G.MODEL_DECODER)
    load_weights(m, w)
    if delta is not None:
        m.write_graft("weight", delta)
    return m


@pytest.mark.parametrize("domain_id", [1, 3])
def test_overlay_forward_matches_oracle(domain_id):
    rc = ov_cfg(domain_id=domain_id)
    B, T = 2, 128
    w, delta, ids, _ = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T)
    logits = m.forward(ids.cuda())
    energies = [m.activation(5, l, torch.float32).cpu() for l in range(rc.num_layers)]
    torch.cuda.synchronize()
    ref_logits, ref_x, _, saves = rm.model_forward(ids, w, delta, rc)
    for l in range(rc.num_layers):
        assert_close_bf16(m.activation(3, l).float().cpu(), saves[l]["x_post"].reshape(-1), f"x_post L{l}")
        M = B * T
        for p, key, width in ((0, "delta_gate", rc.slice_dim), (1, "delta_up", rc.slice_dim),
                              (2, "delta_down", rc.h_slice_dim)):
            want = saves[l][key].pow(2).sum(-1)
            assert_close_bf16(energies[l][p * M:(p + 1) * M], want, f"energy sum L{l} p{p}")
    assert_close_bf16(m.activation(0, rc.num_layers).float().cpu(), ref_x.reshape(-1), "final residual")
    assert_close_bf16(logits.float().cpu(), ref_logits.reshape(-1, rc.vocab_size), "logits")
    m.close()


@pytest.mark.parametrize("projs", [(0, 0, 1), (1, 0, 1), (0, 1, 0), (1, 1, 1)])
def test_overlay_train_step_matches_oracle(projs, wide=False):
    over = dict(graft_proj_gate=projs[0], graft_proj_up=projs[1], graft_proj_down=projs[2])
    if wide:
        # H = 2048 / 4 = 512: the weight-grad GEMMs take 128x256 tiles
        over.update(hidden_dim=2048, num_heads=16, num_kv_heads=4, intermediate_dim=1024, slice_dim=256,
                    num_layers=1, graft_layer_end=0)
    rc = ov_cfg(**over)
    B, T = 4, 128
    w, delta, ids, ood = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T)
    st = m.train_step(ids, ood, step=0, total_steps=10)
    grad_gpu = m.read_graft("grad").cpu()
    w_gpu = m.read_graft("weight").cpu()
    m.close()
    grad_ref, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), rc)
    assert st["lm_loss"] == pytest.approx(stats["lm_loss"], rel=1e-2)
    assert st["silence_loss"] == pytest.approx(stats["silence"], rel=2e-2)
    assert st["total_loss"] == pytest.approx(stats["total_loss"], rel=1e-2)
    assert st["domain_graft_energy"] == pytest.approx(stats["domain_energy"], rel=2e-2)
    assert st["ood_graft_energy"] == pytest.approx(stats["ood_energy"], rel=2e-2)
    SH = rc.slice_dim * rc.h_slice_dim
    for l in range(rc.num_layers):
        for p, name in enumerate(("gate", "up", "down")):
            sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
            if not rc.should_graft_proj(l, p):
                assert float(grad_gpu[sl].abs().max()) == 0.0
                continue
            # overlay grads are nonzero for every enabled projection
            assert float(grad_ref[sl].abs().max()) > 0
            assert_close_bf16(grad_gpu[sl], grad_ref[sl], f"grad L{l} {name}")
    norm_ref = (float(grad_ref.double().pow(2).sum()) + 1e-8) ** 0.5
    assert st["grad_norm"] == pytest.approx(norm_ref, rel=1e-2)
    w_ref = delta.clone()
    g2 = grad_gpu.clone()
    rm.clip_grads(g2, rc.gradient_clip_norm)
    rm.adamw(w_ref, g2, torch.zeros_like(w_ref), torch.zeros_like(w_ref), 0, rc.get_lr(0, 10), rc)
    torch.testing.assert_close(w_gpu, w_ref, rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("projs", [(1, 1, 1), (0, 0, 1)])
def test_overlay_train_step_wide_h_slice(projs):
    test_overlay_train_step_matches_oracle(projs, wide=True)


def test_overlay_layer_range_and_base_only_forward():
    rc = ov_cfg(graft_layer_start=1, graft_layer_end=1)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T)
    base = m.forward(ids.cuda(), use_graft=False).float().cpu()
    grafted = m.forward(ids.cuda(), use_graft=True).float().cpu()
    m.close()
    ref_base, _, _, _ = rm.model_forward(ids, w, None, rc)
    ref_graft, _, _, _ = rm.model_forward(ids, w, delta, rc)
    assert_close_bf16(base, ref_base.reshape(-1, rc.vocab_size), "base logits")
    assert_close_bf16(grafted, ref_graft.reshape(-1, rc.vocab_size), "grafted logits")


def test_overlay_shadow_bake_is_bit_exact_and_within_bake_budget():
    rc = ov_cfg(graft_proj_gate=1, graft_proj_up=0, graft_proj_down=1, domain_id=2)
    B, T = 2, 128
    w, delta, ids, _ = problem(rc, B, T, graft_std=0.02)
    m = gpu_model(rc, w, delta, B, T)
    explicit = m.eval(ids, use_graft=True)
    base = m.eval(ids, use_graft=False)
    m.shadow_bake()
    shadow = m.eval(ids, use_graft=False)
    m.close()
    # G2: baked == explicit within the bf16 bake budget, and closer to the
    # explicit graft than the unbaked base is
    assert abs(shadow["mean_ce"] - explicit["mean_ce"]) < 0.02
    assert shadow["logits_hash"] != base["logits_hash"]
    assert abs(shadow["logits_sum"] - explicit["logits_sum"]) < abs(base["logits_sum"] - explicit["logits_sum"])
    assert shadow["graft_forward_calls"] == 0
    # the oracle's bit-exact bake (shadow_bake_impl.inc:15-128) of the same weights,
    # loaded as a plain base model, gives the identical logits fingerprint
    layers = [dict(gate=bx.f32_to_bf16_bits(lw["wg"].numpy()), up=bx.f32_to_bf16_bits(lw["wu"].numpy()),
                   down=bx.f32_to_bf16_bits(lw["wd"].numpy())) for lw in w["layers"]]
    bx.apply_graft_to_shadow(layers, delta.numpy(), rc, bx.ShadowBakeState(), rc.domain_id)
    wb = dict(w)
    wb["layers"] = []
    for lw, bl in zip(w["layers"], layers):
        d = dict(lw)
        d["wg"] = torch.from_numpy(bx.bf16_bits_to_f32(bl["gate"]).copy())
        d["wu"] = torch.from_numpy(bx.bf16_bits_to_f32(bl["up"]).copy())
        d["wd"] = torch.from_numpy(bx.bf16_bits_to_f32(bl["down"]).copy())
        wb["layers"].append(d)
    m2 = gpu_model(rc, wb, None, B, T)
    ref = m2.eval(ids, use_graft=False)
    m2.close()
    assert ref["logits_hash"] == shadow["logits_hash"]
    assert ref["mean_ce"] == shadow["mean_ce"]


def test_overlay_mlp_block_step_matches_oracle():
    from glt_b200 import graft as G
    rc = rm.GraftConfig(hidden_dim=256, intermediate_dim=640, slice_dim=160, max_domains=4,
                        domain_id=1, num_layers=1, vocab_size=0, num_heads=4, num_kv_heads=4,
                        graft_layer_start=0, graft_layer_end=0, graft_proj_gate=1, graft_proj_up=0,
                        graft_proj_down=1, layout="overlay", adam_weight_decay=0.0).finalize()
    M = 256
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, rc.hidden_dim, generator=g).to(torch.bfloat16).float()
    y = torch.randn(M, rc.hidden_dim, generator=g)
    w = make_decoder_weights(rc, 1, 0.02)
    lw = w["layers"][0]
    delta = torch.randn(3 * rc.slice_dim * rc.h_slice_dim, generator=g) * 0.02
    m = G.GraftModel(to_glt_config(rc), 2, 128, kind=G.MODEL_MLP_BLOCK)
    load_weights(m, w, decoder=False)
    m.write_graft("weight", delta)
    out = m.block_step(x, y, lr=1e-4, step=0)
    grad = m.read_graft("grad").cpu()
    m.close()
    ref = rm.mlp_block_step(x, y, lw, delta.clone(), torch.zeros_like(delta),
                            torch.zeros_like(delta), rc, 1e-4)
    assert_close_bf16(out["out"].float().cpu(), ref["out"], "block out")
    assert out["loss"] == pytest.approx(ref["loss"], rel=1e-2)
    assert_close_bf16(grad, ref["grad"], "block graft grads")
    assert_close_bf16(out["dx"].float().cpu(), ref["dx"], "block dx")
