"""Stored MLP activations (glt_model_mlp_store): the training forward keeps
bf16 gate_pre/up and the backward fuses SwiGLU's backward into the dh GEMM,
against the recompute path (the reference's recompute_ffn,
src/layer_recompute_impl.inc:8-91) and the fp32 oracle, in both
geometries.  Both backward epilogue widths run: concat F' = 896
(128-column tiles) and F' = 1152 (256-column tiles, the last one half
full); overlay F' = 768 and 1024 with slices off the 32-column grid."""
import pytest
import torch

from oracle import ref_math as rm
from tests.parity import assert_close_bf16, load_weights, make_decoder_weights, rel_cos, to_glt_config

pytestmark = pytest.mark.gpu

RECOMPUTE, STORE, AUTO, QUERY = 0, 1, 2, -1


def cfg(**over):
    kw = dict(hidden_dim=256, intermediate_dim=640, slice_dim=128, vocab_size=512, num_layers=2,
              num_heads=4, num_kv_heads=2, rope_theta=10000.0, graft_layer_start=0,
              graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
              layout="concat", lambda_silence=5.0, tie_embeddings=True)
    kw.update(over)
    return rm.GraftConfig(**kw).finalize()


def problem(rc, B, T, seed=0, std=0.05, graft_std=0.05):
    w = make_decoder_weights(rc, seed, std)
    g = torch.Generator().manual_seed(seed + 100)
    delta = torch.randn(rc.total_projections * rc.slice_dim * rc.h_slice_dim, generator=g) * graft_std
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=g, dtype=torch.int32)
    ood = (torch.rand(B, T, generator=g) < 0.4).to(torch.int32)
    return w, delta, ids, ood


def gpu_model(rc, w, delta, B, T, mode):
    from glt_b200 import graft as G
    m = G.GraftModel(to_glt_config(rc), B, T, kind=G.MODEL_DECODER)
    load_weights(m, w)
    m.write_graft("weight", delta)
    m.mlp_store(mode)
    return m


def store_bytes(rc, B, T):
    F_pad = -(-rc.intermediate_dim // 256) * 256
    S_pad = -(-rc.slice_dim // 128) * 128
    FF = F_pad if rc.layout == "overlay" else F_pad + S_pad
    per = B * T * 2 * FF * 2
    return rc.num_layers * (-(-per // 256) * 256)


def test_store_modes():
    rc = cfg()
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T, AUTO)
    assert m.mlp_store(QUERY) == (False, 0)          # auto: nothing before a training step
    m.train_step(ids, ood, 0, 4)
    assert m.mlp_store(QUERY) == (True, store_bytes(rc, B, T))
    assert m.mlp_store(RECOMPUTE) == (False, 0)
    m.train_step(ids, ood, 1, 4)
    assert m.mlp_store(QUERY) == (False, 0)
    assert m.mlp_store(STORE) == (True, store_bytes(rc, B, T))
    from glt_b200._lib import GltError
    with pytest.raises(GltError):
        m.mlp_store(3)
    m.close()


@pytest.mark.parametrize("inter,S,dom,projs", [
    (640, 40, 1, (1, 1, 1)),     # slice [40, 80): not on the 32-column chunk grid; 128-wide dh tiles
    (640, 40, 1, (0, 0, 1)),
    (640, 160, 1, (1, 0, 1)),
    (1024, 16, 3, (1, 1, 1)),    # slice [48, 64), 256-wide dh tiles
])
def test_overlay_store_matches_recompute_and_oracle(inter, S, dom, projs):
    """The reference's own geometry: the forward stores gate_pre/up after the
    delta injection, the dh GEMM's epilogue adds the ContractInputGrad slice
    and writes the silence-blended expand grads and the h slice."""
    rc = cfg(layout="overlay", max_domains=4, domain_id=dom, intermediate_dim=inter, slice_dim=S,
             graft_proj_gate=projs[0], graft_proj_up=projs[1], graft_proj_down=projs[2])
    B, T = 4, 128
    w, delta, ids, ood = problem(rc, B, T)
    runs = {}
    for mode in (RECOMPUTE, AUTO):
        m = gpu_model(rc, w, delta, B, T, mode)
        st = m.train_step(ids, ood, step=0, total_steps=10)
        assert m.mlp_store(QUERY) == ((True, store_bytes(rc, B, T)) if mode == AUTO else (False, 0))
        runs[mode] = (st, m.read_graft("grad").cpu())
        m.close()
    (s0, g0), (s1, g1) = runs[RECOMPUTE], runs[AUTO]
    for k in ("lm_loss", "silence_loss", "domain_graft_energy", "ood_graft_energy"):
        assert s1[k] == pytest.approx(s0[k], rel=1e-5, abs=1e-9), k
    grad_ref, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), rc)
    assert s1["total_loss"] == pytest.approx(stats["total_loss"], rel=1e-2)
    SH = rc.slice_dim * rc.h_slice_dim
    for l in range(rc.num_layers):
        for p, name in enumerate(("gate", "up", "down")):
            sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
            if not rc.should_graft_proj(l, p):
                assert float(g1[sl].abs().max()) == 0.0
                continue
            assert_close_bf16(g1[sl], grad_ref[sl], f"stored overlay: grad L{l} {name}")
            assert_close_bf16(g1[sl], g0[sl], f"stored vs recompute overlay: grad L{l} {name}")
    assert s1["grad_norm"] == pytest.approx(s0["grad_norm"], rel=1e-2)


@pytest.mark.parametrize("inter", [640, 1024])
@pytest.mark.parametrize("projs", [(1, 1, 1), (1, 0, 1), (0, 0, 1)])
def test_store_matches_recompute_and_oracle(inter, projs):
    rc = cfg(intermediate_dim=inter, graft_proj_gate=projs[0], graft_proj_up=projs[1],
             graft_proj_down=projs[2])
    B, T = 4, 128
    w, delta, ids, ood = problem(rc, B, T)
    runs = {}
    for mode in (RECOMPUTE, STORE):
        m = gpu_model(rc, w, delta, B, T, mode)
        st = m.train_step(ids, ood, step=0, total_steps=10)
        assert m.mlp_store(QUERY)[0] == (mode == STORE)
        runs[mode] = (st, m.read_graft("grad").cpu(), m.read_graft("weight").cpu())
        m.close()
    (s0, g0, _), (s1, g1, w1) = runs[RECOMPUTE], runs[STORE]
    # the forward runs the same kernels in both modes; its sums use fp32
    # atomics, so the losses and energies agree to rounding
    for k in ("lm_loss", "silence_loss", "domain_graft_energy", "ood_graft_energy"):
        assert s1[k] == pytest.approx(s0[k], rel=1e-5, abs=1e-9), k
    grad_ref, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), rc)
    assert s1["total_loss"] == pytest.approx(stats["total_loss"], rel=1e-2)
    SH = rc.slice_dim * rc.h_slice_dim
    for l in range(rc.num_layers):
        for p, name in enumerate(("gate", "up", "down")):
            sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
            if float(grad_ref[sl].abs().max()) == 0.0:
                assert float(g1[sl].abs().max()) == 0.0
                continue
            assert_close_bf16(g1[sl], grad_ref[sl], f"stored: grad L{l} {name}")
            assert_close_bf16(g1[sl], g0[sl], f"stored vs recompute: grad L{l} {name}")
    assert s1["grad_norm"] == pytest.approx(s0["grad_norm"], rel=1e-2)
    # clip + AdamW on the stored path's own gradients
    w_ref = delta.clone()
    g2 = g1.clone()
    rm.clip_grads(g2, rc.gradient_clip_norm)
    rm.adamw(w_ref, g2, torch.zeros_like(w_ref), torch.zeros_like(w_ref), 0, rc.get_lr(0, 10), rc)
    torch.testing.assert_close(w1, w_ref, rtol=1e-5, atol=1e-8)


def test_store_several_steps_track_recompute():
    """Four AdamW steps: the two backward paths give the same loss curve and
    the same direction of the graft update (AdamW's early updates are close to
    lr * sign(g), so elementwise they are ill-conditioned across two gradient
    sources; the cosine is not)."""
    rc = cfg(intermediate_dim=1024, lr_peak=5e-3, lr_warmup_steps=1)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T, std=0.02, graft_std=0.02)
    out = {}
    for mode in (RECOMPUTE, STORE):
        m = gpu_model(rc, w, delta, B, T, mode)
        losses = [m.train_step(ids.cuda(), ood.cuda(), s, 4)["total_loss"] for s in range(4)]
        out[mode] = (losses, m.read_graft("weight").cpu())
        m.close()
    for a, b in zip(out[RECOMPUTE][0], out[STORE][0]):
        assert b == pytest.approx(a, rel=2e-3)
    assert out[STORE][0][-1] < out[STORE][0][0]
    _, cos = rel_cos(out[STORE][1] - delta, out[RECOMPUTE][1] - delta)
    assert cos >= 0.99, f"graft update direction after 4 steps: cos {cos:.4f}"
