"""Parity at the geometries the benchmarks run, against the fp32 CPU oracle.

The other decoder tests use small shapes (hidden 256/512, 4 heads, 128-256
tokens).  These run the measured layer geometries themselves, two layers
deep, so that the paths small shapes cannot reach are checked:

* Llama-3-8B layer (the training benchmark): hidden 4096, base intermediate
  14336 + graft 1024, 32 query / 8 KV heads of 128, 2 x 2048 tokens (32
  m-tiles: one full raster group of the persistent GEMM), with the stored
  MLP pre-activations and with the reference's recompute (recompute_ffn,
  src/layer_recompute_impl.inc:8-91).  The vocabulary is cut to 32768 rows
  to bound the oracle's CPU time and memory; the LM-head GEMMs only see
  fewer N tiles.
* Qwen2.5-0.5B layer: hidden 896 (not a multiple of 256), 14 query / 2 KV
  heads (GQA ratio 7), head_dim 64, intermediate 4864 + graft 512, tied
  embeddings over the full 151936-token vocabulary, 2 x 1024 tokens.
* LM-head chunking: 6 x 2048 tokens with a random OOD mask, so the live-row
  LM head runs one full 8192-row chunk and a partial one, and the GEMMs run
  three raster groups with a partial last one.

The bar is the bf16 gate of tests/parity.py (norm-relative max error <= 2e-2,
cosine >= 0.999 against fp32).  With GLT_PARITY_LOG set to a file path,
every compared tensor appends one JSON line {test, tensor, rel, cos} there.
"""
import json
import os

import pytest
import torch

from oracle import ref_math as rm
from tests.parity import assert_close_bf16, load_weights, make_decoder_weights, to_glt_config

pytestmark = pytest.mark.gpu

RECOMPUTE, STORE = 0, 1


def check(got, ref, what, test):
    rel, cos = assert_close_bf16(got, ref, f"{test}: {what}")
    path = os.environ.get("GLT_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(dict(test=test, tensor=what, rel=rel, cos=cos)) + "\n")


def geometry(name):
    if name == "llama3_8b_layer":
        return dict(rc=dict(hidden_dim=4096, intermediate_dim=14336, slice_dim=1024, vocab_size=32768,
                            num_heads=32, num_kv_heads=8, head_dim=128, rope_theta=500000.0,
                            tie_embeddings=False),
                    B=2, T=2048, std=0.02, graft_std=0.02, mask="halves")
    if name == "qwen25_05b_layer":
        return dict(rc=dict(hidden_dim=896, intermediate_dim=4864, slice_dim=512, vocab_size=151936,
                            num_heads=14, num_kv_heads=2, head_dim=64, rope_theta=1000000.0,
                            tie_embeddings=True),
                    B=2, T=1024, std=0.02, graft_std=0.02, mask="halves")
    if name == "lm_head_chunks":
        return dict(rc=dict(hidden_dim=256, intermediate_dim=640, slice_dim=128, vocab_size=512,
                            num_heads=4, num_kv_heads=2, head_dim=64, rope_theta=10000.0,
                            tie_embeddings=False),
                    B=6, T=2048, std=0.05, graft_std=0.05, mask="random")
    raise KeyError(name)


def build(name):
    g = geometry(name)
    rc = rm.GraftConfig(num_layers=2, graft_layer_start=0, graft_layer_end=1, graft_proj_gate=1,
                        graft_proj_up=1, graft_proj_down=1, layout="concat", lambda_silence=5.0,
                        **g["rc"]).finalize()
    B, T = g["B"], g["T"]
    w = make_decoder_weights(rc, seed=3, std=g["std"])
    gen = torch.Generator().manual_seed(103)
    delta = torch.randn(rc.total_projections * rc.slice_dim * rc.h_slice_dim, generator=gen) * g["graft_std"]
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=gen, dtype=torch.int32)
    if g["mask"] == "halves":     # the reference's batch layout (grafting.hip:965-983)
        ood = torch.zeros(B, T, dtype=torch.int32)
        ood[B // 2:] = 1
    else:
        ood = (torch.rand(B, T, generator=gen) < 0.4).to(torch.int32)
    return rc, B, T, w, delta, ids, ood


_ORACLE = {}


def oracle(name):
    """Oracle forward + explicit backward of one step, computed once per geometry."""
    if name not in _ORACLE:
        rc, B, T, w, delta, ids, ood = build(name)
        torch.set_num_threads(os.cpu_count() or 1)
        keep = {}
        grad, stats, logits = rm.compute_grads(ids, ood, w, delta.clone(), rc, keep=keep)
        _ORACLE[name] = dict(problem=(rc, B, T, w, delta, ids, ood),
                             logits=logits.detach().reshape(-1, rc.vocab_size), acts=keep["acts"],
                             grad=grad, stats=stats)
    return _ORACLE[name]


def run_gpu(name, mode):
    from glt_b200 import graft as G
    o = oracle(name)
    rc, B, T, w, delta, ids, ood = o["problem"]
    m = G.GraftModel(to_glt_config(rc), B, T, kind=G.MODEL_DECODER)
    try:
        load_weights(m, w)
        m.write_graft("weight", delta)
        active, _ = m.mlp_store(mode)
        assert active == (mode == STORE)
        logits = m.forward(ids.cuda())
        torch.cuda.synchronize()
        acts = [dict(x_post=m.activation(3, l).float().cpu(), x_ffn=m.activation(4, l).float().cpu())
                for l in range(rc.num_layers)]
        logits = logits.float().cpu()
        st = m.train_step(ids, ood, step=0, total_steps=10)
        grad = m.read_graft("grad").cpu()
    finally:
        m.close()
    return rc, o, acts, logits, st, grad


def compare(name, mode):
    rc, o, acts, logits, st, grad = run_gpu(name, mode)
    test = f"{name}/{'store' if mode == STORE else 'recompute'}"
    for l in range(rc.num_layers):
        check(acts[l]["x_post"], o["acts"][l]["x_post"], f"x_post L{l}", test)
        check(acts[l]["x_ffn"], o["acts"][l]["x_ffn"], f"x_ffn L{l}", test)
    check(logits, o["logits"], "logits", test)
    ref = o["stats"]
    assert st["lm_loss"] == pytest.approx(ref["lm_loss"], rel=1e-2)
    assert st["silence_loss"] == pytest.approx(ref["silence"], rel=2e-2)
    assert st["total_loss"] == pytest.approx(ref["total_loss"], rel=1e-2)
    assert st["domain_graft_energy"] == pytest.approx(ref["domain_energy"], rel=2e-2)
    assert st["ood_graft_energy"] == pytest.approx(ref["ood_energy"], rel=2e-2)
    SH = rc.slice_dim * rc.h_slice_dim
    for l in range(rc.num_layers):
        for p, pname in enumerate(("gate", "up", "down")):
            sl = slice((3 * l + p) * SH, (3 * l + p + 1) * SH)
            check(grad[sl], o["grad"][sl], f"grad L{l} {pname}", test)
    norm_ref = (float(o["grad"].double().pow(2).sum()) + 1e-8) ** 0.5
    assert st["grad_norm"] == pytest.approx(norm_ref, rel=1e-2)


@pytest.mark.parametrize("mode", [STORE, RECOMPUTE])
def test_llama3_8b_layer_geometry(mode):
    compare("llama3_8b_layer", mode)


@pytest.mark.parametrize("mode", [STORE, RECOMPUTE])
def test_qwen25_05b_layer_geometry(mode):
    compare("qwen25_05b_layer", mode)


def test_lm_head_chunks_and_raster_groups():
    compare("lm_head_chunks", STORE)
