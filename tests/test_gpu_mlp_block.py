"""The single-block workload on the GPU: one pre-RMSNorm grafted MLP block
(hidden 256, base intermediate 688 + graft 64 concatenated), MSE loss,
backward to the graft only, one AdamW step -- against the fp32 oracle."""
import pytest
import torch

from oracle import ref_math as rm
from tests.parity import assert_close_bf16, bf16r, to_glt_config

pytestmark = pytest.mark.gpu


def build(graft_down_std: float, M: int = 256, D: int = 256, F: int = 688, S: int = 64, seed: int = 0):
    rc = rm.GraftConfig(hidden_dim=D, intermediate_dim=F, slice_dim=S, num_layers=1, num_heads=4,
                        num_kv_heads=4, vocab_size=0, graft_layer_start=0, graft_layer_end=0,
                        graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1, layout="concat",
                        adam_weight_decay=0.0, lambda_silence=0.0).finalize()
    g = torch.Generator().manual_seed(seed)
    x = bf16r(torch.randn(M, D, generator=g))
    y = torch.randn(M, D, generator=g)
    lw = dict(post_norm=torch.ones(D), wg=bf16r(torch.randn(F, D, generator=g) * 0.02),
              wu=bf16r(torch.randn(F, D, generator=g) * 0.02),
              wd=bf16r(torch.randn(D, F, generator=g) * 0.02))
    H = D
    delta = torch.zeros(3 * S * H)
    delta[:S * H] = torch.randn(S * H, generator=g) * 0.02
    delta[S * H:2 * S * H] = torch.randn(S * H, generator=g) * 0.02
    if graft_down_std:
        delta[2 * S * H:] = torch.randn(S * H, generator=g) * graft_down_std
    return rc, x, y, lw, delta


def run_gpu(rc, x, y, lw, delta, lr, M):
    from glt_b200 import graft as G
    cfg = to_glt_config(rc)
    m = G.GraftModel(cfg, 1, M, kind=G.MODEL_MLP_BLOCK)
    m.set_weight(0, G.W_POST_NORM, lw["post_norm"])
    m.set_weight(0, G.W_GATE, lw["wg"])
    m.set_weight(0, G.W_UP, lw["wu"])
    m.set_weight(0, G.W_DOWN, lw["wd"])
    m.write_graft("weight", delta)
    r = m.block_step(x, y, lr=lr, step=0)
    torch.cuda.synchronize()
    r["grad"] = m.read_graft("grad").cpu()
    r["weight"] = m.read_graft("weight").cpu()
    m.close()
    return r


@pytest.mark.parametrize("down_std", [0.0, 0.02])
def test_config1_block_step(down_std):
    M, S, D = 256, 64, 256
    rc, x, y, lw, delta = build(down_std, M=M)
    lr = 1e-4
    gpu = run_gpu(rc, x, y, lw, delta.clone(), lr, M)
    w = delta.clone()
    m0, v0 = torch.zeros_like(w), torch.zeros_like(w)
    ref = rm.mlp_block_step(x, y, lw, w, m0, v0, rc, lr=lr)
    assert gpu["loss"] == pytest.approx(ref["loss"], rel=1e-2)
    assert_close_bf16(gpu["out"].float().cpu(), ref["out"], "block output")
    assert_close_bf16(gpu["dx"].cpu(), ref["dx"], "input grad")
    SH = S * D
    g_gpu, g_ref = gpu["grad"], ref["grad"]
    assert_close_bf16(g_gpu[2 * SH:], g_ref[2 * SH:], "graft down grad")
    if down_std == 0.0:
        # zero-init down: gate/up get exactly zero gradient, so AdamW leaves them unchanged
        assert float(g_gpu[:2 * SH].abs().max()) == 0.0
        assert torch.equal(gpu["weight"][:2 * SH], delta[:2 * SH])
    else:
        assert_close_bf16(g_gpu[:SH], g_ref[:SH], "graft gate grad")
        assert_close_bf16(g_gpu[SH:2 * SH], g_ref[SH:2 * SH], "graft up grad")
    # AdamW: the oracle optimizer applied to the GPU's own gradients gives the
    # GPU's updated weights (comparing updates across two gradient sources is
    # ill-conditioned at step 0, where the update is ~lr * sign(g)).
    w2 = delta.clone()
    rm.adamw(w2, g_gpu.clone(), torch.zeros_like(w2), torch.zeros_like(w2), 0, lr, rc)
    torch.testing.assert_close(gpu["weight"], w2, rtol=1e-5, atol=1e-8)


def test_config5_shape_small_m():
    """C5 microbench geometry (hidden 4096, base 14336, graft 256) at a small token count."""
    M, D, F, S = 256, 4096, 14336, 256
    rc, x, y, lw, delta = build(0.02, M=M, D=D, F=F, S=S, seed=1)
    gpu = run_gpu(rc, x, y, lw, delta.clone(), 1e-4, M)
    w = delta.clone()
    ref = rm.mlp_block_step(x, y, lw, w, torch.zeros_like(w), torch.zeros_like(w), rc, lr=1e-4)
    assert_close_bf16(gpu["out"].float().cpu(), ref["out"], "C5 block output")
    assert_close_bf16(gpu["dx"].cpu(), ref["dx"], "C5 input grad")
    assert_close_bf16(gpu["grad"], ref["grad"], "C5 graft grads")
