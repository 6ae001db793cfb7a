"""fp32 CPU restatement of the reference's grafted decoder training step.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA library;
only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import it.  The product path never calls it.

It follows Hinedes/GLT's algorithm function by function, in fp32 on the
CPU (torch), for both graft geometries:
  * "overlay" -- the reference's own semantics: deltas are added into the
    axis-aligned slice [i0, i0+S) x [h0, h0+H) of the base projections
    (src/layer_forward_impl.inc:21-22);
  * "concat"  -- the [base | graft] intermediate layout the benchmarks use:
    overlay on a base zero-padded from F to F+S with i0 = F, h0 = 0, H = D.
The MLP backward is the reference's explicit backward
(src/layer_backward_impl.inc:10-385); attention backward re-runs the forward
under autograd exactly as src/attention_autograd_impl.inc:1-39 does.

Parity of the orientation conventions is pinned by the reference's golden
vectors (tests/test_oracle_golden.py); the floating-point path itself is
checked against torch autograd of the same loss (tests/test_oracle_math.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2


# ---------------------------------------------------------------------------
# Configuration (src/config.hpp:40-129, grafting.hip:274-400)
# ---------------------------------------------------------------------------
@dataclass
class GraftConfig:
    hidden_dim: int = 2048
    intermediate_dim: int = 11008
    slice_dim: int = 2752
    vocab_size: int = 128256
    num_layers: int = 36
    num_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 0
    max_domains: int = 4
    domain_id: int = 0
    rms_norm_eps: float = 1e-6
    lm_loss_scale: float = 1.0
    lambda_silence: float = 5.0
    rope_theta: float = 5000000.0
    no_rope_layers: list = field(default_factory=list)
    graft_layer_start: int = 0
    graft_layer_end: int = 35
    graft_proj_gate: int = 0
    graft_proj_up: int = 0
    graft_proj_down: int = 1
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_eps: float = 1e-8
    adam_weight_decay: float = 0.01
    gradient_clip_norm: float = 1.0
    lr_warmup_steps: int = 20
    lr_peak: float = 2e-4
    layout: str = "overlay"      # "overlay" (reference) or "concat" ([base | graft])
    tie_embeddings: bool = True

    def finalize(self) -> "GraftConfig":
        if self.head_dim == 0:
            self.head_dim = self.hidden_dim // self.num_heads
        return self

    # geometry ---------------------------------------------------------------
    @property
    def h_slice_dim(self) -> int:
        if self.layout == "concat":
            return self.hidden_dim
        return self.hidden_dim // self.max_domains

    @property
    def i0(self) -> int:
        return self.intermediate_dim if self.layout == "concat" else self.domain_id * self.slice_dim

    @property
    def h0(self) -> int:
        return 0 if self.layout == "concat" else self.domain_id * self.h_slice_dim

    @property
    def ffn_dim(self) -> int:
        """Width of the intermediate activation (F, or F+S for concat)."""
        return self.intermediate_dim + (self.slice_dim if self.layout == "concat" else 0)

    @property
    def total_projections(self) -> int:
        return 3 * self.num_layers

    def should_graft_layer(self, l: int) -> bool:      # src/config.hpp:100-102
        return self.graft_layer_start <= l <= self.graft_layer_end

    def should_graft_proj(self, l: int, p: int) -> bool:  # src/config.hpp:104-110
        if not self.should_graft_layer(l):
            return False
        return bool((self.graft_proj_gate, self.graft_proj_up, self.graft_proj_down)[p])

    def count_active_grafts(self) -> int:              # src/config.hpp:112-120
        return sum(self.should_graft_proj(l, p) for l in range(self.num_layers) for p in range(3))

    def rope_enabled(self, l: int) -> bool:            # src/layer_forward_impl.inc:37
        return (not self.no_rope_layers) or bool(self.no_rope_layers[l])

    def get_lr(self, step: int, total_steps: int) -> float:  # src/config.hpp:122-129
        from .bitexact import get_lr
        return get_lr(step, total_steps, self.lr_peak, self.lr_warmup_steps)


def delta_view(delta: torch.Tensor, cfg: GraftConfig, l: int, p: int) -> torch.Tensor:
    """[S,H] view of projection p of layer l in the flat buffer (src/graft_ops_impl.inc:5-7)."""
    S, H = cfg.slice_dim, cfg.h_slice_dim
    off = (l * 3 + p) * S * H
    return delta.view(-1)[off:off + S * H].view(S, H)


# ---------------------------------------------------------------------------
# Building blocks
# ---------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float):
    """Returns (y, variance); kernels_rmsnorm_kernels.inc:8-60."""
    var = x.pow(2).mean(-1)
    y = x * torch.rsqrt(var + eps).unsqueeze(-1) * w
    return y, var


def rms_norm_bwd(dy, x, w, var, eps):
    """kernels_rmsnorm_kernels.inc:70-126: dx = dy*r*w - x*mean(dy*x*w)*r^3."""
    r = torch.rsqrt(var + eps).unsqueeze(-1)
    mean_term = (dy * x * w).mean(-1, keepdim=True)
    return dy * r * w - x * mean_term * r.pow(3)


def rope_tables(seq_len: int, head_dim: int, theta: float):
    """rope_impl.inc:13-19: inv_freq = 1/theta^(i/hd), emb = cat(angles, angles)."""
    i = torch.arange(0, head_dim, 2, dtype=torch.float32)
    inv_freq = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float32), i / head_dim)
    pos = torch.arange(seq_len, dtype=torch.float32)
    ang = pos.unsqueeze(-1) * inv_freq.unsqueeze(0)
    emb = torch.cat([ang, ang], -1)
    return emb.cos(), emb.sin()


def apply_rope(t: torch.Tensor, nh: int, hd: int, cos, sin):
    """Half-split rotation (rope_impl.inc:21-36); t is [B, T, nh*hd]."""
    B, T, _ = t.shape
    v = t.view(B, T, nh, hd)
    half = hd // 2
    x1, x2 = v[..., :half], v[..., half:]
    c = cos.view(1, T, 1, hd)
    s = sin.view(1, T, 1, hd)
    r1 = x1 * c[..., :half] - x2 * s[..., :half]
    r2 = x2 * c[..., half:] + x1 * s[..., half:]
    return torch.cat([r1, r2], -1).view(B, T, nh * hd)


def causal_gqa_attention(q, k, v, nh, nkv, hd):
    """layer_forward_impl.inc:41-49: repeat_interleave GQA, causal SDPA."""
    B, T, _ = q.shape
    rep = nh // nkv
    qh = q.view(B, T, nh, hd).transpose(1, 2)
    kh = k.view(B, T, nkv, hd).transpose(1, 2).repeat_interleave(rep, 1)
    vh = v.view(B, T, nkv, hd).transpose(1, 2).repeat_interleave(rep, 1)
    scores = (qh @ kh.transpose(-1, -2)) / math.sqrt(hd)
    mask = torch.ones(T, T, dtype=torch.bool).tril()
    scores = scores.masked_fill(~mask, float("-inf"))
    o = torch.softmax(scores, -1) @ vh
    return o.transpose(1, 2).reshape(B, T, nh * hd)


def attention_block(x, lw, cfg: GraftConfig, l: int):
    """x + o_proj(attn(rope(q), rope(k), v)) of rms_norm(x) (layer_forward_impl.inc:25-52)."""
    B, T, D = x.shape
    xn, _ = rms_norm(x, lw["in_norm"], cfg.rms_norm_eps)
    q = xn @ lw["wq"].t()
    k = xn @ lw["wk"].t()
    v = xn @ lw["wv"].t()
    if cfg.rope_enabled(l):
        cos, sin = rope_tables(T, cfg.head_dim, cfg.rope_theta)
        q = apply_rope(q, cfg.num_heads, cfg.head_dim, cos, sin)
        k = apply_rope(k, cfg.num_kv_heads, cfg.head_dim, cos, sin)
    a = causal_gqa_attention(q, k, v, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim)
    return x + a @ lw["wo"].t()


# ---------------------------------------------------------------------------
# Grafted MLP
# ---------------------------------------------------------------------------
def base_mlp_weights(lw, cfg: GraftConfig):
    """Base gate/up [F', D] and down [D, F'] with F' = F (+S zero rows/cols for concat)."""
    wg, wu, wd = lw["wg"], lw["wu"], lw["wd"]
    if cfg.layout == "concat":
        S, D = cfg.slice_dim, cfg.hidden_dim
        z = torch.zeros(S, D, dtype=wg.dtype)
        wg = torch.cat([wg, z], 0)
        wu = torch.cat([wu, z], 0)
        wd = torch.cat([wd, z.t()], 1)
    return wg, wu, wd


def energy(delta: torch.Tensor, width: int, eps: float = 1e-8) -> torch.Tensor:
    """sqrt(sum(delta^2) + eps) / sqrt(width) per token (kernels_elementwise_impl.inc:287-367)."""
    return torch.sqrt(delta.pow(2).sum(-1) + eps) / math.sqrt(max(width, 1))


def mlp_forward(x_ffn: torch.Tensor, lw, delta: torch.Tensor | None, cfg: GraftConfig, l: int):
    """Grafted SwiGLU MLP forward (layer_forward_impl.inc:61-218).

    x_ffn: [M, D] normalised input.  Returns (ffn_out [M, D], saved dict).
    """
    S, H, i0, h0 = cfg.slice_dim, cfg.h_slice_dim, cfg.i0, cfg.h0
    M = x_ffn.shape[0]
    wg, wu, wd = base_mlp_weights(lw, cfg)
    x_h = x_ffn[:, h0:h0 + H]
    saved = {}
    gp = x_ffn @ wg.t()
    up = x_ffn @ wu.t()
    for p, t in ((PROJ_GATE, gp), (PROJ_UP, up)):
        key = "gate" if p == PROJ_GATE else "up"
        if delta is not None and cfg.should_graft_proj(l, p):
            d = x_h @ delta_view(delta, cfg, l, p).t()          # ExpandForward [M, S]
            t[:, i0:i0 + S] += d
            saved["delta_" + key] = d
            saved["energy_" + key] = energy(d, S)
        else:
            saved["delta_" + key] = torch.zeros(M, S)
            saved["energy_" + key] = torch.zeros(M)
    h = torch.nn.functional.silu(gp) * up
    ffn = h @ wd.t()
    if delta is not None and cfg.should_graft_proj(l, PROJ_DOWN):
        d = h[:, i0:i0 + S] @ delta_view(delta, cfg, l, PROJ_DOWN)  # ContractForward [M, H]
        ffn[:, h0:h0 + H] += d
        saved["delta_down"] = d
        saved["energy_down"] = energy(d, H)
    else:
        saved["delta_down"] = torch.zeros(M, H)
        saved["energy_down"] = torch.zeros(M)
    return ffn, saved


def mlp_backward(dy: torch.Tensor, x_ffn: torch.Tensor, lw, delta: torch.Tensor, saved,
                 cfg: GraftConfig, l: int, ood: torch.Tensor, lambda_eff: float,
                 grad: torch.Tensor):
    """Explicit backward of the grafted MLP (layer_backward_impl.inc:36-361).

    dy: [M, D] gradient wrt ffn_out.  Writes graft weight grads into `grad`
    (flat [3L*S*H], overwrite semantics, layer_backward via beta=0) and
    returns dx_ffn [M, D].
    """
    S, H, i0, h0 = cfg.slice_dim, cfg.h_slice_dim, cfg.i0, cfg.h0
    wg, wu, wd = base_mlp_weights(lw, cfg)
    # recompute_ffn (layer_recompute_impl.inc:8-91), fp32
    gp = x_ffn @ wg.t()
    up = x_ffn @ wu.t()
    if cfg.should_graft_proj(l, PROJ_GATE):
        gp[:, i0:i0 + S] += saved["delta_gate"]
    if cfg.should_graft_proj(l, PROJ_UP):
        up[:, i0:i0 + S] += saved["delta_up"]
    sg = torch.sigmoid(gp)
    h = gp * sg * up
    # Step 1: base down
    gi = dy @ wd
    # Step 2: contract delta + silence on OOD tokens (silence_blend_kernel, :8-67)
    if cfg.should_graft_proj(l, PROJ_DOWN):
        dyh = dy[:, h0:h0 + H].clone()
        dd = saved["delta_down"]
        norm = torch.sqrt(dd.pow(2).sum(-1) + 1e-8)
        scale = lambda_eff / (norm * math.sqrt(H))
        dyh += (ood.float() * scale).unsqueeze(-1) * dd
        delta_view(grad, cfg, l, PROJ_DOWN).copy_(h[:, i0:i0 + S].t() @ dyh)
        gi[:, i0:i0 + S] += dyh @ delta_view(delta, cfg, l, PROJ_DOWN).t()
    # Step 3: SwiGLU backward (fused_gate_up_bwd_kernel, :80-124)
    dgp = gi * up * sg * (1.0 + gp * (1.0 - sg))
    dup = gi * gp * sg
    # Steps 4+5: expand deltas with fused silence (fused_silence_blend_energy_kernel, :458-560)
    grad_x_h = torch.zeros(dy.shape[0], H)
    x_h = x_ffn[:, h0:h0 + H]
    if cfg.should_graft_proj(l, PROJ_GATE) or cfg.should_graft_proj(l, PROJ_UP):
        for p, src, key in ((PROJ_GATE, dgp, "delta_gate"), (PROJ_UP, dup, "delta_up")):
            if not cfg.should_graft_proj(l, p):
                continue
            dys = src[:, i0:i0 + S].clone()
            dlt = saved[key]
            e = energy(dlt, S)
            norm = e * math.sqrt(S)
            scale = lambda_eff / (norm * math.sqrt(S) + 1e-8)
            dys += (ood.float() * scale).unsqueeze(-1) * dlt
            delta_view(grad, cfg, l, p).copy_(dys.t() @ x_h)           # ExpandWeightGrad
            grad_x_h += dys @ delta_view(delta, cfg, l, p)             # ExpandInputGrad
    # Step 6: base gate/up input grad
    dx = dgp @ wg + dup @ wu
    dx[:, h0:h0 + H] += grad_x_h
    return dx


# ---------------------------------------------------------------------------
# Decoder layer / model
# ---------------------------------------------------------------------------
def layer_forward(x, lw, delta, cfg: GraftConfig, l: int):
    """forward_layer (layer_forward_impl.inc:15-291); x: [B, T, D]."""
    B, T, D = x.shape
    x_pre = x
    x_post = attention_block(x, lw, cfg, l)
    x_ffn, var = rms_norm(x_post, lw["post_norm"], cfg.rms_norm_eps)
    ffn, saved = mlp_forward(x_ffn.reshape(B * T, D), lw, delta, cfg, l)
    saved.update(x_pre=x_pre, x_post=x_post, x_ffn=x_ffn.reshape(B * T, D), var=var)
    return x_post + ffn.view(B, T, D), saved


def layer_backward(dx, lw, delta, saved, cfg: GraftConfig, l: int, ood_flat, lambda_eff, grad):
    """backward_layer (layer_backward_impl.inc:10-385); dx: [B, T, D] grad of layer output."""
    B, T, D = dx.shape
    dffn = mlp_backward(dx.reshape(B * T, D), saved["x_ffn"], lw, delta, saved, cfg, l,
                        ood_flat, lambda_eff, grad)
    g_norm = rms_norm_bwd(dffn.view(B, T, D), saved["x_post"], lw["post_norm"], saved["var"],
                          cfg.rms_norm_eps)
    g_post_total = dx + g_norm
    # attention_bwd_autograd (attention_autograd_impl.inc:1-39)
    xa = saved["x_pre"].detach().clone().requires_grad_(True)
    with torch.enable_grad():
        y = attention_block(xa, lw, cfg, l)
        y.backward(g_post_total)
    return xa.grad.detach()


def model_forward(ids, weights, delta, cfg: GraftConfig):
    """forward_model (grafting.hip:224-271). ids: [B, T] int."""
    x = weights["embed"][ids.long()]
    saves = []
    for l in range(cfg.num_layers):
        x, s = layer_forward(x, weights["layers"][l], delta, cfg, l)
        saves.append(s)
    xn, var = rms_norm(x, weights["final_norm"], cfg.rms_norm_eps)
    logits = xn @ weights["lm_head"].t()
    return logits, x, var, saves


def lm_loss_and_grad(logits, ids, ood, cfg: GraftConfig):
    """CE over domain tokens and its gradient (grafting.hip:1027-1042, 1122-1135)."""
    B, T, V = logits.shape
    labels = ids[:, 1:].long().reshape(-1)
    lg = logits[:, :-1].reshape(-1, V)
    logp = torch.log_softmax(lg, -1)
    ce = -logp.gather(-1, labels.unsqueeze(-1)).squeeze(-1)
    dmask = (1 - ood[:, 1:].reshape(-1)).float()
    in_count = max(float(dmask.sum()), 1.0)
    loss = (ce * dmask).sum() / in_count
    probs = torch.softmax(lg, -1)
    probs[torch.arange(labels.numel()), labels] -= 1.0
    g = probs * dmask.unsqueeze(-1) / in_count * cfg.lm_loss_scale
    dlogits = torch.zeros_like(logits)
    dlogits[:, :-1] = g.view(B, T - 1, V)
    return float(loss), dlogits, in_count


def silence_terms(saves, ood, cfg: GraftConfig):
    """Silence loss and lambda_eff (grafting.hip:1053-1106)."""
    ood_f = ood.reshape(-1).float()
    dom_f = 1.0 - ood_f
    ood_count = float(ood_f.sum())
    dom_count = max(float((1 - ood[:, 1:]).sum()), 1.0)
    active = cfg.count_active_grafts()
    stats = dict(silence=0.0, domain_energy=0.0, ood_energy=0.0, ratio=0.0, lambda_eff=0.0)
    if ood_count > 0 and dom_count > 0 and active > 0:
        dacc = 0.0
        oacc = 0.0
        for l, s in enumerate(saves):
            for p, key in ((0, "energy_gate"), (1, "energy_up"), (2, "energy_down")):
                if cfg.should_graft_proj(l, p):
                    dacc += float((s[key] * dom_f).sum()) / dom_count
                    oacc += float((s[key] * ood_f).sum()) / ood_count
        dacc /= active
        oacc /= active
        stats.update(domain_energy=dacc, ood_energy=oacc,
                     ratio=(dacc / oacc) if oacc > 0 else 0.0,
                     silence=cfg.lambda_silence * oacc,
                     lambda_eff=cfg.lambda_silence / (ood_count * active))
    return stats


def clip_grads(grad: torch.Tensor, clip: float):
    """reduce_l2 -> calc_scale -> apply_scale (kernels_elementwise_impl.inc:133-213)."""
    norm = math.sqrt(float(grad.double().pow(2).sum()) + 1e-8)
    scale = clip / norm if norm > clip else 1.0
    grad.mul_(scale)
    return norm, scale


def adamw(weight, grad, m, v, step: int, lr: float, cfg: GraftConfig):
    """adamw_fused_kernel + execute_adamw_all (kernels_optimizer_impl.inc:11-77).

    Masked projection kinds are skipped entirely (:23-28); the layer range is
    not consulted here, exactly as in the reference.
    """
    b1, b2 = cfg.adam_beta1, cfg.adam_beta2
    c1 = 1.0 / (1.0 - b1 ** (step + 1))
    c2 = 1.0 / (1.0 - b2 ** (step + 1))
    S, H = cfg.slice_dim, cfg.h_slice_dim
    enabled = (cfg.graft_proj_gate, cfg.graft_proj_up, cfg.graft_proj_down)
    for proj in range(cfg.total_projections):
        if not enabled[proj % 3]:
            continue
        sl = slice(proj * S * H, (proj + 1) * S * H)
        g = grad.view(-1)[sl]
        mm = m.view(-1)[sl]
        vv = v.view(-1)[sl]
        w = weight.view(-1)[sl]
        mm.mul_(b1).add_((1 - b1) * g)
        vv.mul_(b2).add_((1 - b2) * g * g)
        upd = lr * (mm * c1) / (torch.sqrt(vv * c2) + cfg.adam_eps) + lr * cfg.adam_weight_decay * w
        w.sub_(upd)


def compute_grads(ids, ood, weights, delta, cfg: GraftConfig, keep=None):
    """Forward, loss, silence and the explicit backward of one step (grafting.hip:997-1146).

    Returns (grad [flat, pre-clip], stats dict, logits).  `keep`, a dict, if
    given receives per layer the forward's x_post and x_ffn ([M*D] each).
    """
    logits, x_last, var_f, saves = model_forward(ids, weights, delta, cfg)
    if keep is not None:
        keep["acts"] = [dict(x_post=s["x_post"].detach().reshape(-1).clone(),
                             x_ffn=s["x_ffn"].detach().reshape(-1).clone()) for s in saves]
    loss, dlogits, _ = lm_loss_and_grad(logits, ids, ood, cfg)
    sil = silence_terms(saves, ood, cfg)
    dx = dlogits @ weights["lm_head"]
    dx = rms_norm_bwd(dx, x_last, weights["final_norm"], var_f, cfg.rms_norm_eps)
    grad = torch.zeros_like(delta)
    ood_flat = ood.reshape(-1)
    for l in reversed(range(cfg.num_layers)):
        dx = layer_backward(dx, weights["layers"][l], delta, saves[l], cfg, l, ood_flat,
                            sil["lambda_eff"], grad)
    stats = dict(lm_loss=loss, total_loss=cfg.lm_loss_scale * loss + sil["silence"], **sil)
    return grad, stats, logits


def train_step(ids, ood, weights, delta, m, v, cfg: GraftConfig, step: int, total_steps: int):
    """One training step (grafting.hip:954-1172).  Mutates delta, m, v.

    Returns a dict with losses, the pre-clip grad norm, the clipped grads and
    the logits.
    """
    grad, stats, logits = compute_grads(ids, ood, weights, delta, cfg)
    norm, scale = clip_grads(grad, cfg.gradient_clip_norm)
    lr = cfg.get_lr(step, total_steps)
    adamw(delta, grad, m, v, step, lr, cfg)
    return dict(grad_norm=norm, clip_scale=scale, grad=grad, logits=logits, lr=lr, **stats)


# ---------------------------------------------------------------------------
# Single grafted MLP block (hidden 256, base 688 + graft 64 workload)
# ---------------------------------------------------------------------------
def mlp_block_step(x, y, lw, delta, m, v, cfg: GraftConfig, lr: float, step: int = 0):
    """Pre-RMSNorm grafted MLP block with residual, MSE loss, graft-only AdamW.

    out = x + MLP(rms_norm(x)); loss = mean((out - y)^2).  Reuses the
    reference's MLP forward/backward (no OOD tokens -> no silence term).
    Returns dict(out, loss, grad, dx).
    """
    M, D = x.shape
    xn, var = rms_norm(x, lw["post_norm"], cfg.rms_norm_eps)
    ffn, saved = mlp_forward(xn, lw, delta, cfg, 0)
    out = x + ffn
    loss = float((out - y).pow(2).mean())
    dy = 2.0 * (out - y) / out.numel()
    grad = torch.zeros_like(delta)
    dffn = mlp_backward(dy, xn, lw, delta, saved, cfg, 0, torch.zeros(M, dtype=torch.int32), 0.0,
                        grad)
    dx = dy + rms_norm_bwd(dffn, x, lw["post_norm"], var, cfg.rms_norm_eps)
    adamw(delta, grad, m, v, step, lr, cfg)
    return dict(out=out, loss=loss, grad=grad, dx=dx, saved=saved)


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (N(0, 0.02) weights)
# ---------------------------------------------------------------------------
def init_weights(cfg: GraftConfig, seed: int = 0, std: float = 0.02):
    g = torch.Generator().manual_seed(seed)
    D, F = cfg.hidden_dim, cfg.intermediate_dim
    nh, nkv, hd, V = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.vocab_size

    def rn(*s):
        return torch.randn(*s, generator=g) * std

    layers = []
    for _ in range(cfg.num_layers):
        layers.append(dict(in_norm=torch.ones(D), wq=rn(nh * hd, D), wk=rn(nkv * hd, D),
                           wv=rn(nkv * hd, D), wo=rn(D, nh * hd), post_norm=torch.ones(D),
                           wg=rn(F, D), wu=rn(F, D), wd=rn(D, F)))
    embed = rn(V, D) if V > 0 else None
    lm_head = embed if cfg.tie_embeddings else (rn(V, D) if V > 0 else None)
    return dict(embed=embed, lm_head=lm_head, final_norm=torch.ones(D), layers=layers)


def silu_product(gate_pre: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """fused_silu_product_strided_kernel (kernels_elementwise_impl.inc:411-448):
    bf16(gp * sigmoid(gp) * up) from bf16 operands, fp32 math."""
    g, u = gate_pre.float(), up.float()
    return (g * torch.sigmoid(g) * u).to(torch.bfloat16)


def gate_up_backward(grad_h: torch.Tensor, up: torch.Tensor, gate_pre: torch.Tensor):
    """fused_gate_up_bwd_kernel (kernels_elementwise_impl.inc:80-124):
    sg = sigmoid(gp); grad_gate_pre = gi * up * sg * (1 + gp * (1 - sg));
    grad_up = gi * gp * sg (fp32 outputs)."""
    g, u, gi = gate_pre.float(), up.float(), grad_h.float()
    sg = torch.sigmoid(g)
    return gi * u * (sg * (1 + g * (1 - sg))), gi * (g * sg)


# ---------------------------------------------------------------------------
# Graft stacks: sibling grafts of several domains active at once
# ---------------------------------------------------------------------------
def mlp_forward_stack(x_ffn: torch.Tensor, lw, deltas: list, cfg: GraftConfig, l: int):
    """MLP forward with the grafts of domains 0..N-1 injected explicitly, each
    into its own overlay slice (i0 = d*S, h0 = d*H): path A of
    tests/test6_stack_vs_bake_f32.cpp:66-163 (gate and up deltas added to the
    pre-activations, silu(gate)*up, base down GEMM, down deltas added to the
    output), extended from two domains to N and from one MLP to a layer."""
    S, H = cfg.slice_dim, cfg.hidden_dim // cfg.max_domains
    wg, wu, wd = lw["wg"], lw["wu"], lw["wd"]
    gp = x_ffn @ wg.t()
    up = x_ffn @ wu.t()
    for d, delta in enumerate(deltas):
        i0, h0 = d * S, d * H
        x_h = x_ffn[:, h0:h0 + H]
        if cfg.should_graft_proj(l, PROJ_GATE):
            gp[:, i0:i0 + S] += x_h @ delta_view_at(delta, cfg, l, PROJ_GATE, S, H).t()
        if cfg.should_graft_proj(l, PROJ_UP):
            up[:, i0:i0 + S] += x_h @ delta_view_at(delta, cfg, l, PROJ_UP, S, H).t()
    h = torch.nn.functional.silu(gp) * up
    ffn = h @ wd.t()
    for d, delta in enumerate(deltas):
        i0, h0 = d * S, d * H
        if cfg.should_graft_proj(l, PROJ_DOWN):
            ffn[:, h0:h0 + H] += h[:, i0:i0 + S] @ delta_view_at(delta, cfg, l, PROJ_DOWN, S, H)
    return ffn


def delta_view_at(delta: torch.Tensor, cfg: GraftConfig, l: int, p: int, S: int, H: int):
    """[S, H] view of projection (l, p) of a flat [3L, S, H] graft (delta_offset)."""
    off = (l * 3 + p) * S * H
    return delta.view(-1)[off:off + S * H].view(S, H)


def model_forward_stack(ids, weights, deltas: list, cfg: GraftConfig):
    """forward_model (grafting.hip:224-271) with a stack of N domain grafts,
    each injected explicitly (mlp_forward_stack).  Returns logits [B, T, V]."""
    x = weights["embed"][ids.long()]
    B, T, D = x.shape
    for l in range(cfg.num_layers):
        lw = weights["layers"][l]
        x_post = attention_block(x, lw, cfg, l)
        x_ffn, _ = rms_norm(x_post, lw["post_norm"], cfg.rms_norm_eps)
        x = x_post + mlp_forward_stack(x_ffn.reshape(B * T, D), lw, deltas, cfg, l).view(B, T, D)
    xn, _ = rms_norm(x, weights["final_norm"], cfg.rms_norm_eps)
    return xn @ weights["lm_head"].t()


def stack_grafts(deltas: list, num_layers: int, S: int, H: int) -> torch.Tensor:
    """N sibling grafts [3L, S, H] -> one [3L, N*S, N*H] graft whose
    projection blocks are block-diagonal (domain d at rows [dS, (d+1)S) and
    columns [dH, (d+1)H)).  As one overlay graft at i0 = h0 = 0 it computes
    exactly the N explicit injections (the off-diagonal zeros add nothing)
    and bakes to the same base (bf16(base + 0) == base)."""
    N = len(deltas)
    out = torch.zeros(3 * num_layers, N * S, N * H, dtype=torch.float32)
    for d, delta in enumerate(deltas):
        out[:, d * S:(d + 1) * S, d * H:(d + 1) * H] = delta.view(3 * num_layers, S, H)
    return out.view(-1)
