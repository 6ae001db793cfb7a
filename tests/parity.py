"""Shared helpers of the parity tests: the bf16 tolerance of the north star and
seeded problem builders that feed identical inputs to the CUDA path and to
the fp32 CPU oracle."""
from __future__ import annotations

import torch

# bf16 tolerance vs the fp32 oracle (the reference's bf16 error-budget gate):
# norm-relative max error <= 2e-2 and cosine similarity >= 0.999.
MAX_REL = 2e-2
MIN_COS = 0.999


def rel_cos(got: torch.Tensor, ref: torch.Tensor):
    g = got.detach().double().cpu().reshape(-1)
    r = ref.detach().double().cpu().reshape(-1)
    denom = float(r.abs().max())
    rel = float((g - r).abs().max()) / denom if denom > 0 else float((g - r).abs().max())
    nn = float(g.norm() * r.norm())
    cos = float((g @ r) / nn) if nn > 0 else (1.0 if float(g.abs().max()) == 0 else 0.0)
    return rel, cos


def assert_close_bf16(got, ref, what: str, max_rel: float = MAX_REL, min_cos: float = MIN_COS):
    rel, cos = rel_cos(got, ref)
    assert rel <= max_rel and cos >= min_cos, f"{what}: max rel {rel:.3e} (<= {max_rel}), cos {cos:.6f} (>= {min_cos})"
    return rel, cos


def bf16r(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and back (the values the GPU path stores)."""
    return t.to(torch.bfloat16).float()


def make_decoder_weights(cfg, seed: int, std: float = 0.02):
    """HF-shaped fp32 weights, already bf16-rounded, for an oracle GraftConfig."""
    g = torch.Generator().manual_seed(seed)
    D, F = cfg.hidden_dim, cfg.intermediate_dim
    nh, nkv, hd, V = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.vocab_size

    def rn(*s):
        return bf16r(torch.randn(*s, generator=g) * std)

    layers = []
    for _ in range(cfg.num_layers):
        layers.append(dict(in_norm=torch.ones(D), wq=rn(nh * hd, D), wk=rn(nkv * hd, D),
                           wv=rn(nkv * hd, D), wo=rn(D, nh * hd), post_norm=torch.ones(D),
                           wg=rn(F, D), wu=rn(F, D), wd=rn(D, F)))
    embed = rn(V, D) if V else None
    return dict(embed=embed, lm_head=embed if cfg.tie_embeddings else rn(V, D),
                final_norm=torch.ones(D), layers=layers)


def load_weights(model, w, decoder: bool = True):
    from glt_b200 import graft as G
    if decoder:
        model.set_weight(-1, G.W_EMBED, w["embed"])
        model.set_weight(-1, G.W_LM_HEAD, w["lm_head"])
        model.set_weight(-1, G.W_FINAL_NORM, w["final_norm"])
    for l, lw in enumerate(w["layers"]):
        if decoder:
            model.set_weight(l, G.W_IN_NORM, lw["in_norm"])
            model.set_weight(l, G.W_Q, lw["wq"])
            model.set_weight(l, G.W_K, lw["wk"])
            model.set_weight(l, G.W_V, lw["wv"])
            model.set_weight(l, G.W_O, lw["wo"])
        model.set_weight(l, G.W_POST_NORM, lw["post_norm"])
        model.set_weight(l, G.W_GATE, lw["wg"])
        model.set_weight(l, G.W_UP, lw["wu"])
        model.set_weight(l, G.W_DOWN, lw["wd"])


def to_glt_config(rc, **over):
    """oracle.ref_math.GraftConfig -> glt_b200.graft.GraftConfig."""
    from glt_b200 import graft as G
    kw = dict(hidden_dim=rc.hidden_dim, intermediate_dim=rc.intermediate_dim, slice_dim=rc.slice_dim,
              vocab_size=rc.vocab_size, num_layers=rc.num_layers, num_heads=rc.num_heads,
              num_kv_heads=rc.num_kv_heads, head_dim=rc.head_dim, max_domains=rc.max_domains,
              domain_id=rc.domain_id, layout=G.LAYOUT_CONCAT if rc.layout == "concat" else G.LAYOUT_OVERLAY,
              tie_embeddings=int(rc.tie_embeddings), rms_norm_eps=rc.rms_norm_eps,
              lm_loss_scale=rc.lm_loss_scale, lambda_silence=rc.lambda_silence, rope_theta=rc.rope_theta,
              graft_layer_start=rc.graft_layer_start, graft_layer_end=rc.graft_layer_end,
              graft_proj_gate=rc.graft_proj_gate, graft_proj_up=rc.graft_proj_up,
              graft_proj_down=rc.graft_proj_down, allow_expansion_trap=1,
              adam_beta1=rc.adam_beta1, adam_beta2=rc.adam_beta2, adam_eps=rc.adam_eps,
              adam_weight_decay=rc.adam_weight_decay, gradient_clip_norm=rc.gradient_clip_norm,
              lr_warmup_steps=rc.lr_warmup_steps, lr_peak=rc.lr_peak,
              no_rope_layers=list(rc.no_rope_layers))
    kw.update(over)
    return G.GraftConfig(**kw)
