"""Checks the fp32 oracle's floating-point path (CPU only).

* the explicit (reference-structured) backward equals torch autograd of the
  same loss -- LM cross-entropy on domain tokens + silence on OOD tokens --
  in both graft geometries;
* concat geometry equals overlay on a zero-padded base (the identity the
  [base | graft] layout relies on);
* explicit graft injection equals the baked model in fp32
  (tests/test6_stack_vs_bake_f32.cpp semantics, with its inputs).
"""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import ref_math as rm

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def tiny_cfg(layout, gate=1, up=1, down=1):
    c = rm.GraftConfig(hidden_dim=32, intermediate_dim=48, slice_dim=16, vocab_size=50,
                       num_layers=2, num_heads=4, num_kv_heads=2, max_domains=2, domain_id=1,
                       rope_theta=10000.0, graft_layer_start=0, graft_layer_end=1,
                       graft_proj_gate=gate, graft_proj_up=up, graft_proj_down=down,
                       lambda_silence=5.0, layout=layout, lm_loss_scale=1.0)
    return c.finalize()


def random_problem(cfg, seed=0, B=4, T=8):
    torch.manual_seed(seed)
    w = rm.init_weights(cfg, seed=seed, std=0.2)
    for lw in w["layers"]:
        lw["in_norm"] = 1.0 + 0.1 * torch.randn(cfg.hidden_dim)
        lw["post_norm"] = 1.0 + 0.1 * torch.randn(cfg.hidden_dim)
    delta = torch.randn(cfg.total_projections * cfg.slice_dim * cfg.h_slice_dim) * 0.2
    ids = torch.randint(0, cfg.vocab_size, (B, T), dtype=torch.int32)
    ood = torch.zeros(B, T, dtype=torch.int32)
    ood[B // 2:] = 1
    return w, delta, ids, ood


def autograd_loss(ids, ood, w, delta, cfg):
    logits, _, _, saves = rm.model_forward(ids, w, delta, cfg)
    B, T, V = logits.shape
    labels = ids[:, 1:].long().reshape(-1)
    logp = torch.log_softmax(logits[:, :-1].reshape(-1, V), -1)
    ce = -logp.gather(-1, labels.unsqueeze(-1)).squeeze(-1)
    dmask = (1 - ood[:, 1:].reshape(-1)).float()
    in_count = max(float(dmask.sum()), 1.0)
    loss = (ce * dmask).sum() / in_count
    oodf = ood.reshape(-1).float()
    oc = float(oodf.sum())
    acc = 0.0
    for l, s in enumerate(saves):
        for p, k in ((0, "energy_gate"), (1, "energy_up"), (2, "energy_down")):
            if cfg.should_graft_proj(l, p):
                acc = acc + (s[k] * oodf).sum() / oc
    acc = acc / cfg.count_active_grafts()
    return cfg.lm_loss_scale * loss + cfg.lambda_silence * acc


@pytest.mark.parametrize("layout", ["overlay", "concat"])
@pytest.mark.parametrize("projs", [(1, 1, 1), (0, 0, 1), (1, 0, 0)])
def test_explicit_backward_matches_autograd(layout, projs):
    cfg = tiny_cfg(layout, *projs)
    w, delta, ids, ood = random_problem(cfg)
    grad, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), cfg)
    d = delta.clone().requires_grad_(True)
    loss = autograd_loss(ids, ood, w, d, cfg)
    loss.backward()
    assert stats["total_loss"] == pytest.approx(float(loss), rel=1e-5)
    torch.testing.assert_close(grad, d.grad, rtol=1e-4, atol=1e-6)


def test_concat_equals_overlay_on_zero_padded_base():
    cc = tiny_cfg("concat")
    w, delta, ids, ood = random_problem(cc, seed=3)
    logits_c, _, _, _ = rm.model_forward(ids, w, delta, cc)
    # overlay on an explicitly padded base with i0 = F, h0 = 0, H = D
    oc = rm.GraftConfig(**{**cc.__dict__, "layout": "overlay"})
    oc.intermediate_dim = cc.intermediate_dim + cc.slice_dim
    oc.max_domains = 1
    oc.domain_id = 0
    F, S, D = cc.intermediate_dim, cc.slice_dim, cc.hidden_dim
    wp = {**w, "layers": []}
    for lw in w["layers"]:
        z = torch.zeros(S, D)
        wp["layers"].append({**lw, "wg": torch.cat([lw["wg"], z]), "wu": torch.cat([lw["wu"], z]),
                             "wd": torch.cat([lw["wd"], z.t()], 1)})
    # overlay uses i0 = domain*S = 0: move the padded rows to the front instead
    for lw in wp["layers"]:
        lw["wg"] = torch.roll(lw["wg"], S, 0)
        lw["wu"] = torch.roll(lw["wu"], S, 0)
        lw["wd"] = torch.roll(lw["wd"], S, 1)
    logits_o, _, _, _ = rm.model_forward(ids, wp, delta, oc)
    torch.testing.assert_close(logits_c, logits_o, rtol=1e-5, atol=1e-5)


def test_stack_vs_bake_f32_reference_inputs():
    k = KATS["stack_vs_bake_f32"]
    S, H, D, F, M = k["S"], k["H"], k["D"], k["F"], k["M"]
    gate = torch.tensor([(i + 1) * 0.1 for i in range(F * D)]).view(F, D)
    up = torch.tensor([(i + 1) * 0.07 for i in range(F * D)]).view(F, D)
    down = torch.tensor([(i + 1) * 0.05 for i in range(D * F)]).view(D, F)
    x = torch.tensor(k["x"], dtype=torch.float32).view(M, D)

    def mk(b, stp):
        return torch.tensor([[b + i * stp + j for j in range(H)] for i in range(S)])

    g = [mk(*k["gate"][0]), mk(*k["gate"][1])]
    u = [mk(*k["up"][0]), mk(*k["up"][1])]
    dn = [mk(*k["down"][0]), mk(*k["down"][1])]
    # path A: explicit injection of both domains via the oracle's overlay MLP
    lw = dict(wg=gate, wu=up, wd=down)
    outs = []
    ffn_a = None
    cfg = rm.GraftConfig(hidden_dim=D, intermediate_dim=F, slice_dim=S, max_domains=2,
                         num_layers=1, graft_layer_end=0, graft_proj_gate=1, graft_proj_up=1,
                         graft_proj_down=1).finalize()
    # inject domain 0 and domain 1 deltas: sum of two overlays == one forward with both slices
    gp = x @ gate.t()
    upv = x @ up.t()
    for dom in (0, 1):
        gp[:, dom * S:(dom + 1) * S] += x[:, dom * H:(dom + 1) * H] @ g[dom].t()
        upv[:, dom * S:(dom + 1) * S] += x[:, dom * H:(dom + 1) * H] @ u[dom].t()
    h = torch.nn.functional.silu(gp) * upv
    ffn_a = h @ down.t()
    for dom in (0, 1):
        ffn_a[:, dom * H:(dom + 1) * H] += h[:, dom * S:(dom + 1) * S] @ dn[dom]
    # path B: bake both, single forward
    gb, ub, db = gate.clone(), up.clone(), down.clone()
    for dom in (0, 1):
        gb[dom * S:(dom + 1) * S, dom * H:(dom + 1) * H] += g[dom]
        ub[dom * S:(dom + 1) * S, dom * H:(dom + 1) * H] += u[dom]
        db[dom * H:(dom + 1) * H, dom * S:(dom + 1) * S] += dn[dom].t()
    ffn_b = (torch.nn.functional.silu(x @ gb.t()) * (x @ ub.t())) @ db.t()
    md = (ffn_a - ffn_b).abs().max()
    ma = torch.maximum(ffn_a.abs(), ffn_b.abs()).max()
    assert md < k["gate_abs"] or md / ma < k["gate_rel"]
    # the oracle's overlay MLP (domain 1 only) agrees with the hand-written path
    cfg.domain_id = 1
    delta = torch.zeros(3 * S * H)
    rm.delta_view(delta, cfg, 0, 0).copy_(g[1])
    rm.delta_view(delta, cfg, 0, 1).copy_(u[1])
    rm.delta_view(delta, cfg, 0, 2).copy_(dn[1])
    ffn_o, _ = rm.mlp_forward(x, lw, delta, cfg, 0)
    gp1 = x @ gate.t()
    up1 = x @ up.t()
    gp1[:, S:2 * S] += x[:, H:2 * H] @ g[1].t()
    up1[:, S:2 * S] += x[:, H:2 * H] @ u[1].t()
    h1 = torch.nn.functional.silu(gp1) * up1
    f1 = h1 @ down.t()
    f1[:, H:2 * H] += h1[:, S:2 * S] @ dn[1]
    torch.testing.assert_close(ffn_o, f1, rtol=1e-6, atol=1e-5)


def test_mlp_block_step_runs_config1_shapes():
    cfg = rm.GraftConfig(hidden_dim=256, intermediate_dim=688, slice_dim=64, num_layers=1,
                         graft_layer_end=0, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                         layout="concat", adam_weight_decay=0.0).finalize()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 256, generator=g)
    y = torch.randn(256, 256, generator=g)
    lw = dict(post_norm=torch.ones(256), wg=torch.randn(688, 256, generator=g) * 0.02,
              wu=torch.randn(688, 256, generator=g) * 0.02, wd=torch.randn(256, 688, generator=g) * 0.02)
    S, H = 64, 256
    delta = torch.zeros(3 * S * H)
    delta[:S * H] = torch.randn(S * H, generator=g) * 0.02
    delta[S * H:2 * S * H] = torch.randn(S * H, generator=g) * 0.02
    m, v = torch.zeros_like(delta), torch.zeros_like(delta)
    r = rm.mlp_block_step(x, y, lw, delta, m, v, cfg, lr=1e-4)
    # zero-init graft down -> graft gate/up receive exactly zero gradient at step 0
    assert float(r["grad"][:2 * S * H].abs().max()) == 0.0
    assert float(r["grad"][2 * S * H:].abs().max()) > 0.0
    assert math.isfinite(r["loss"])


def test_stack_as_block_diagonal_graft_equals_explicit_and_baked():
    """N sibling grafts injected one by one (test6_stack_vs_bake_f32.cpp path A),
    the same grafts as one block-diagonal overlay graft, and the fp32 base with
    all of them baked in (path B) give the same logits (test6 tolerance 1e-4)."""
    from tests.parity import make_decoder_weights
    N, S = 4, 8
    rc = rm.GraftConfig(hidden_dim=64, intermediate_dim=96, slice_dim=S, max_domains=N, vocab_size=64,
                        num_layers=2, num_heads=4, num_kv_heads=2, rope_theta=10000.0,
                        graft_layer_start=0, graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1,
                        graft_proj_down=1, layout="overlay", tie_embeddings=True).finalize()
    H = rc.hidden_dim // N
    w = make_decoder_weights(rc, 3, 0.05)
    g = torch.Generator().manual_seed(7)
    deltas = [torch.randn(3 * rc.num_layers * S * H, generator=g) * 0.05 for _ in range(N)]
    ids = torch.randint(0, rc.vocab_size, (2, 16), generator=g, dtype=torch.int32)
    explicit = rm.model_forward_stack(ids, w, deltas, rc)
    rs = rm.GraftConfig(**{**rc.__dict__, "slice_dim": N * S, "max_domains": 1, "domain_id": 0}).finalize()
    stacked, _, _, _ = rm.model_forward(ids, w, rm.stack_grafts(deltas, rc.num_layers, S, H), rs)
    torch.testing.assert_close(stacked, explicit, rtol=1e-5, atol=1e-5)
    wb = {**w, "layers": []}
    for l, lw in enumerate(w["layers"]):
        lb = {k: v.clone() for k, v in lw.items()}
        for d, delta in enumerate(deltas):
            i0, h0 = d * S, d * H
            lb["wg"][i0:i0 + S, h0:h0 + H] += rm.delta_view_at(delta, rc, l, 0, S, H)
            lb["wu"][i0:i0 + S, h0:h0 + H] += rm.delta_view_at(delta, rc, l, 1, S, H)
            lb["wd"][h0:h0 + H, i0:i0 + S] += rm.delta_view_at(delta, rc, l, 2, S, H).t()
        wb["layers"].append(lb)
    baked, _, _, _ = rm.model_forward(ids, wb, None, rc)
    torch.testing.assert_close(baked, explicit, rtol=1e-4, atol=1e-4)
