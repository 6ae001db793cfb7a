"""Graft stacks (the stacked-inference workload at test size): N sibling grafts of one
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

import numpy as np

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


# ---------------------------------------------------------------------------
# One GRFT file per sibling (glt_model_save_stack / glt_model_load_stack)
# ---------------------------------------------------------------------------
def stack_model(geometry, S_sib=32):
    from oracle import bitexact as bx  # noqa: F401  (parser used by the caller)
    if geometry == "overlay":   # the stack geometry of glt_stack_grafts
        rc = stack_cfg(slice_dim=N * S_sib, max_domains=1, domain_id=0)
    else:
        rc = stack_cfg(slice_dim=N * S_sib, layout="concat", max_domains=4)
    w = make_decoder_weights(rc, 5, 0.02)
    m = G.GraftModel(to_glt_config(rc), 2, 128, kind=G.MODEL_DECODER)
    load_weights(m, w)
    return rc, m


def path_array(paths):
    return (C.c_char_p * len(paths))(*[str(p).encode() for p in paths])


@pytest.mark.parametrize("geometry", ["concat", "overlay"])
def test_stack_files_roundtrip(tmp_path, geometry):
    from oracle import bitexact as bx
    rc, a = stack_model(geometry)
    L, S, H, S_sib = rc.num_layers, rc.slice_dim, rc.h_slice_dim, rc.slice_dim // N
    H_sib = H // N if geometry == "overlay" else H
    g = torch.randn(3 * L * S * H, generator=torch.Generator().manual_seed(3)) * 0.05
    a.write_graft("weight", g)
    paths = [tmp_path / f"sib{d}.graft" for d in range(N)]
    _lib.check(lib.glt_model_save_stack(a.handle, path_array(paths), N, b"sess"))
    full = g.view(3 * L, S, H).numpy()
    want = np.zeros_like(full)
    for d in range(N):
        c0 = d * H_sib if geometry == "overlay" else 0
        blk = full[:, d * S_sib:(d + 1) * S_sib, c0:c0 + H_sib]
        got = bx.parse_grft(open(paths[d], "rb").read(), d, "sess", 3 * L, S_sib, H_sib)
        np.testing.assert_array_equal(np.asarray(got).reshape(blk.shape), bx.round_bf16(blk))
        want[:, d * S_sib:(d + 1) * S_sib, c0:c0 + H_sib] = bx.round_bf16(blk)
    a.close()
    _, b = stack_model(geometry)
    _lib.check(lib.glt_model_load_stack(b.handle, path_array(paths), N, b"sess"))
    np.testing.assert_array_equal(b.read_graft("weight").cpu().numpy().reshape(want.shape), want)
    # refusals leave the graft as it was: siblings out of order (domain ids),
    # a sibling count that does not divide the slice, another session
    before = b.read_graft("weight").cpu()
    for args in ((path_array(paths[::-1]), N, b"sess"), (path_array(paths[:3]), 3, b"sess"),
                 (path_array(paths), N, b"other")):
        with pytest.raises(_lib.GltError):
            _lib.check(lib.glt_model_load_stack(b.handle, *args))
    assert torch.equal(b.read_graft("weight").cpu(), before)
    # the stacked graft is live: the loaded model's forward matches a model given the same values
    c = stack_model(geometry)[1]
    c.write_graft("weight", torch.from_numpy(want).reshape(-1))
    ids = torch.randint(0, rc.vocab_size, (2, 128), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    assert torch.equal(b.forward(ids.cuda()), c.forward(ids.cuda()))
    b.close()
    c.close()
