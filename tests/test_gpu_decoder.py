"""Full grafted decoder step on the GPU against the fp32 oracle: forward
activations layer by layer, logits, LM + silence losses, graft gradients
and the AdamW update, through the C ABI (glt_forward / glt_train_step)."""
import pytest
import torch

from oracle import ref_math as rm
from tests.parity import assert_close_bf16, load_weights, make_decoder_weights, rel_cos, to_glt_config

pytestmark = pytest.mark.gpu


def small_cfg(**over):
    kw = dict(hidden_dim=256, intermediate_dim=640, slice_dim=128, vocab_size=512, num_layers=2,
              num_heads=4, num_kv_heads=2, rope_theta=10000.0, graft_layer_start=0,
              graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
              layout="concat", lambda_silence=5.0, tie_embeddings=True)
    kw.update(over)
    return rm.GraftConfig(**kw).finalize()


def problem(rc, B=2, T=128, seed=0, std=0.02, graft_std=0.02):
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
    m.write_graft("weight", delta)
    return m


@pytest.mark.parametrize("tie", [True, False])
def test_forward_matches_oracle(tie):
    rc = small_cfg(tie_embeddings=tie)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    m = gpu_model(rc, w, delta, B, T)
    logits = m.forward(ids.cuda())
    torch.cuda.synchronize()
    ref_logits, _, _, saves = rm.model_forward(ids, w, delta, rc)
    D = rc.hidden_dim
    for l in range(rc.num_layers):
        assert_close_bf16(m.activation(3, l).float().cpu(), saves[l]["x_post"].reshape(-1), f"x_post L{l}")
        assert_close_bf16(m.activation(4, l).float().cpu(), saves[l]["x_ffn"].reshape(-1), f"x_ffn L{l}")
    assert_close_bf16(logits.float().cpu(), ref_logits.reshape(-1, rc.vocab_size), "logits")
    m.close()


def test_base_forward_skips_graft():
    rc = small_cfg()
    B, T = 2, 128
    w, delta, ids, _ = problem(rc, B, T, graft_std=0.5)
    m = gpu_model(rc, w, delta, B, T)
    lg = m.forward(ids.cuda(), use_graft=False)
    torch.cuda.synchronize()
    ref, _, _, _ = rm.model_forward(ids, w, None, rc)
    assert_close_bf16(lg.float().cpu(), ref.reshape(-1, rc.vocab_size), "base logits")
    m.close()


@pytest.mark.parametrize("projs", [(1, 1, 1), (0, 0, 1)])
def test_train_step_matches_oracle(projs):
    rc = small_cfg(graft_proj_gate=projs[0], graft_proj_up=projs[1], graft_proj_down=projs[2])
    B, T = 4, 128
    w, delta, ids, ood = problem(rc, B, T, std=0.05, graft_std=0.05)
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
            assert_close_bf16(grad_gpu[sl], grad_ref[sl], f"grad L{l} {name}")
    # reference norm: sqrt(sum g^2 + 1e-8) (calc_scale_kernel).  In concat geometry
    # a graft with gate or up disabled has identically zero graft columns, so
    # the down-only case has all-zero gradients in the oracle and on the GPU.
    norm_ref = (float(grad_ref.double().pow(2).sum()) + 1e-8) ** 0.5
    assert st["grad_norm"] == pytest.approx(norm_ref, rel=1e-2)
    if projs != (1, 1, 1):
        assert float(grad_gpu.abs().max()) == 0.0 and float(grad_ref.abs().max()) == 0.0
    # clip + AdamW: the oracle applied to the GPU's own gradients reproduces
    # the GPU's updated weights
    w_ref = delta.clone()
    g2 = grad_gpu.clone()
    rm.clip_grads(g2, rc.gradient_clip_norm)
    rm.adamw(w_ref, g2, torch.zeros_like(w_ref), torch.zeros_like(w_ref), 0, rc.get_lr(0, 10), rc)
    torch.testing.assert_close(w_gpu, w_ref, rtol=1e-5, atol=1e-8)


def test_two_steps_reduce_loss_and_host_inputs_match_device_inputs():
    rc = small_cfg(lr_peak=5e-3, lr_warmup_steps=1)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    m1 = gpu_model(rc, w, delta, B, T)
    s_host = m1.train_step(ids, ood, 0, 4)              # host int32 buffers, copied in the call
    g_host = m1.read_graft("weight").cpu()
    m1.close()
    m2 = gpu_model(rc, w, delta, B, T)
    s_dev = m2.train_step(ids.cuda(), ood.cuda(), 0, 4)  # device buffers
    g_dev = m2.read_graft("weight").cpu()
    losses = [s_dev["total_loss"]]
    for step in range(1, 4):
        losses.append(m2.train_step(ids.cuda(), ood.cuda(), step, 4)["total_loss"])
    m2.close()
    # split-K weight grads and the attention dQ reduction use fp32 atomics, so
    # the two runs agree to rounding, not bit for bit
    assert s_host["total_loss"] == pytest.approx(s_dev["total_loss"], rel=1e-5)
    torch.testing.assert_close(g_host, g_dev, rtol=0, atol=1e-6)
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("mask", ["random", "all_ood", "all_domain"])
def test_train_step_with_any_ood_mask_matches_oracle(mask):
    """The LM head runs only over positions whose next-token label carries LM
    loss (t < T-1 and ood[t+1] == 0, compacted on the device); any mask --
    token-level random, all OOD (no LM rows: the LM-head GEMMs run zero
    tiles) or all domain -- gives the oracle's losses and graft gradients."""
    rc = small_cfg()
    B, T = 4, 128
    w, delta, ids, _ = problem(rc, B, T, std=0.05, graft_std=0.05)
    g = torch.Generator().manual_seed(99)
    if mask == "random":
        ood = (torch.rand(B, T, generator=g) < 0.4).to(torch.int32)
    elif mask == "all_ood":
        ood = torch.ones(B, T, dtype=torch.int32)
    else:
        ood = torch.zeros(B, T, dtype=torch.int32)
    m = gpu_model(rc, w, delta, B, T)
    st = m.train_step(ids, ood, step=0, total_steps=10)
    grad_gpu = m.read_graft("grad").cpu()
    m.close()
    grad_ref, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), rc)
    if mask == "all_ood":
        assert st["lm_loss"] == 0.0 and stats["lm_loss"] == 0.0
    else:
        assert st["lm_loss"] == pytest.approx(stats["lm_loss"], rel=1e-2)
    assert st["total_loss"] == pytest.approx(stats["total_loss"], rel=1e-2, abs=1e-6)
    if float(grad_ref.abs().max()) > 0:
        assert_close_bf16(grad_gpu, grad_ref, f"graft grads ({mask} mask)")
    else:
        assert float(grad_gpu.abs().max()) == 0.0


@pytest.mark.parametrize("no_rope", [[], [1, 0]])
def test_train_step_head_dim_128_matches_oracle(no_rope):
    """head_dim 128 runs the tcgen05 attention backward with the row sums
    D = rowsum(dO o O) from the dO GEMM's epilogue and the inverse RoPE of dq
    in its fp32 -> bf16 conversion (RoPE on layer 0 only with [1, 0])."""
    rc = small_cfg(hidden_dim=512, intermediate_dim=1024, num_heads=4, num_kv_heads=2, no_rope_layers=no_rope)
    assert rc.head_dim == 128
    B, T = 2, 256
    w, delta, ids, ood = problem(rc, B, T, std=0.05, graft_std=0.05)
    m = gpu_model(rc, w, delta, B, T)
    st = m.train_step(ids, ood, step=0, total_steps=10)
    grad_gpu = m.read_graft("grad").cpu()
    m.close()
    grad_ref, stats, _ = rm.compute_grads(ids, ood, w, delta.clone(), rc)
    assert st["lm_loss"] == pytest.approx(stats["lm_loss"], rel=1e-2)
    assert st["total_loss"] == pytest.approx(stats["total_loss"], rel=1e-2)
    SH = rc.slice_dim * rc.h_slice_dim
    for l in range(rc.num_layers):
        for p, name in enumerate(("gate", "up", "down")):
            sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
            assert_close_bf16(grad_gpu[sl], grad_ref[sl], f"hd128 grad L{l} {name}")
