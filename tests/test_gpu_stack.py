"""Graft stacks (BASELINE config 4 at test size): N sibling grafts of one
session active at once, explicitly injected versus shadow-baked.

Overlay geometry (the reference's): domain d's graft sits at intermediate rows
[dS, (d+1)S) and hidden columns [dH, (d+1)H) (layer_forward_impl.inc:21-22).
glt_stack_grafts assembles the N grafts into one block-diagonal graft; its
forward must match the oracle's explicit per-domain injection
(tests/test6_stack_vs_bake_f32.cpp path A) and the shadow-baked model must
agree with the stack within the bf16 gate (max rel <= 2e-2, cos >= 0.999).
Concat geometry: N slices side by side in [base | s_0 | ... | s_{N-1}]; the
bake turns the columns into base columns, so the logits are bit-identical."""
import ctypes as C

import pytest
import torch

from glt_b200 import _lib
from glt_b200 import graft as G
from oracle import ref_math as rm
from tests.parity import assert_close_bf16, load_weights, make_decoder_weights, rel_cos, to_glt_config

pytestmark = pytest.mark.gpu
lib = _lib.lib
N = 4


def stack_cfg(**over):
    kw = dict(hidden_dim=256, intermediate_dim=1024, slice_dim=64, max_domains=N, domain_id=0,
              vocab_size=512, num_layers=2, num_heads=4, num_kv_heads=2, rope_theta=10000.0,
              graft_layer_start=0, graft_layer_end=1, graft_proj_gate=1, graft_proj_up=1,
              graft_proj_down=1, layout="overlay", tie_embeddings=True)
    kw.update(over)
    return rm.GraftConfig(**kw).finalize()


def sibling_grafts(rc, seed=11, std=0.05):
    H = rc.hidden_dim // rc.max_domains
    return [torch.randn(3 * rc.num_layers * rc.slice_dim * H,
                        generator=torch.Generator().manual_seed(seed + d)) * std for d in range(N)]


def gpu_stack(deltas, rc):
    H = rc.hidden_dim // rc.max_domains
    dev = [d.cuda() for d in deltas]
    out = torch.empty(3 * rc.num_layers * N * rc.slice_dim * N * H, device="cuda")
    ptrs = (C.c_void_p * N)(*[t.data_ptr() for t in dev])
    _lib.check(lib.glt_stack_grafts(ptrs, N, rc.num_layers, rc.slice_dim, H, C.c_void_p(out.data_ptr()),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return out


def test_stack_grafts_is_the_block_diagonal_assembly():
    rc = stack_cfg()
    deltas = sibling_grafts(rc)
    got = gpu_stack(deltas, rc).cpu()
    want = rm.stack_grafts(deltas, rc.num_layers, rc.slice_dim, rc.hidden_dim // N)
    assert torch.equal(got, want)


def test_stack_forward_matches_explicit_injection_and_bake_agrees():
    rc = stack_cfg()
    B, T = 2, 128
    w = make_decoder_weights(rc, 5, 0.05)
    deltas = sibling_grafts(rc)
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=torch.Generator().manual_seed(3),
                        dtype=torch.int32)
    rs = rm.GraftConfig(**{**rc.__dict__, "slice_dim": N * rc.slice_dim, "max_domains": 1}).finalize()
    m = G.GraftModel(to_glt_config(rs), B, T, kind=G.MODEL_DECODER)
    load_weights(m, w)
    m.write_graft("weight", gpu_stack(deltas, rc))
    stack = m.forward(ids.cuda(), use_graft=True).float().cpu()
    base = m.forward(ids.cuda(), use_graft=False).float().cpu()
    m.shadow_bake()
    baked = m.forward(ids.cuda(), use_graft=False).float().cpu()
    m.close()
    ref = rm.model_forward_stack(ids, w, deltas, rc).reshape(-1, rc.vocab_size)
    assert_close_bf16(stack, ref, "stack logits vs explicit per-domain injection")
    rel, cos = assert_close_bf16(baked, stack, "baked vs stacked logits")
    # the stack changed the model: the baked logits are nearer the stack than the base is
    rel_base, _ = rel_cos(base, stack)
    assert rel < rel_base


def test_concat_stack_bakes_to_identical_logits():
    S_each = 64
    rc = stack_cfg(layout="concat", slice_dim=N * S_each, max_domains=4)
    B, T = 2, 128
    w = make_decoder_weights(rc, 6, 0.05)
    # N independently seeded slices side by side along the intermediate dimension
    D = rc.hidden_dim
    parts = [torch.randn(3 * rc.num_layers, S_each, D, generator=torch.Generator().manual_seed(40 + d)) * 0.05
             for d in range(N)]
    graft = torch.cat(parts, dim=1).reshape(-1)
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=torch.Generator().manual_seed(4),
                        dtype=torch.int32)
    m = G.GraftModel(to_glt_config(rc), B, T, kind=G.MODEL_DECODER)
    load_weights(m, w)
    m.write_graft("weight", graft)
    stack = m.forward(ids.cuda(), use_graft=True)
    m.shadow_bake()
    baked = m.forward(ids.cuda(), use_graft=False)
    torch.cuda.synchronize()
    m.close()
    assert torch.equal(stack, baked)
    ref, _, _, _ = rm.model_forward(ids, w, graft, rc)
    assert_close_bf16(stack.float().cpu(), ref.reshape(-1, rc.vocab_size), "concat stack vs oracle")
