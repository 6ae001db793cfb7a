"""C ABI surface (CPU only): the library loads without a GPU, exports every
function declared in include/glt_graft.h, and its host-only entry points
follow the reference's rules (defaults, CLI validation, LR schedule, flat
graft layout)."""
import ctypes as C
import os
import re

import pytest

from glt_b200 import _lib
from glt_b200 import graft as G
from oracle import bitexact as bx

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "glt_graft.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"GLT_API\s+[\w\s\*]+?\b(glt_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} not exported by libglt_b200.so"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_version_and_error_string():
    assert b"sm_100a" in _lib.lib.glt_version()
    st = _lib.lib.glt_gemm(None, 0, 0, None, 0, 0, None, 0, 0, 1, 1, 1, 1.0, 0.0, None)
    assert st == 1 and "null" in _lib.last_error()


def test_defaults_match_reference_config():
    d = G.default_config()
    # src/config.hpp:42-90 and grafting.hip:281 (lr)
    assert (d.hidden_dim, d.intermediate_dim, d.slice_dim, d.vocab_size, d.num_layers) == (
        2048, 11008, 2752, 128256, 36)
    assert (d.num_heads, d.num_kv_heads, d.graft_layer_end, d.graft_proj_down) == (16, 4, 35, 1)
    assert (d.graft_proj_gate, d.graft_proj_up) == (0, 0)
    assert d.rms_norm_eps == pytest.approx(1e-6) and d.lambda_silence == 5.0
    assert d.rope_theta == 5e6 and d.adam_weight_decay == pytest.approx(0.01)
    assert d.gradient_clip_norm == 1.0 and d.lr_warmup_steps == 20
    assert d.lr_peak == pytest.approx(2e-4)


@pytest.mark.parametrize("change,msg", [
    (dict(num_heads=0), "num-heads"),
    (dict(max_domains=0), "max-domains"),
    (dict(hidden_dim=2050), "not divisible by num-heads"),
    (dict(hidden_dim=2064, num_heads=8, max_domains=5), "max-domains"),
    (dict(domain_id=4), "out of range"),
    (dict(slice_dim=2750), "not divisible by slice-dim"),
    (dict(graft_proj_down=2), "must be 0 or 1"),
    (dict(graft_proj_down=0), "no graft projection"),
    (dict(graft_proj_gate=1, graft_proj_up=1), "Expansion Quadratic Trap"),
    (dict(no_rope_layers=[1, 0]), "rope-layer-mask"),
])
def test_validation_rules(change, msg):
    c = G.default_config()
    for k, v in change.items():
        setattr(c, k, v)
    with pytest.raises(_lib.GltError) as e:
        c.validate(16)
    assert msg in str(e.value)


def test_validation_batch_must_be_even_for_training_only():
    c = G.default_config()
    with pytest.raises(_lib.GltError):
        c.validate(15, mode=0)
    c.validate(15, mode=1)
    c.graft_proj_gate = c.graft_proj_up = 1
    c.allow_expansion_trap = 1
    c.validate(16)


def test_lr_schedule_matches_oracle():
    c = G.default_config()
    c.lr_peak, c.lr_warmup_steps = 3e-4, 7
    for step in range(0, 60, 3):
        assert c.get_lr(step, 60) == pytest.approx(bx.get_lr(step, 60, 3e-4, 7), rel=1e-6, abs=1e-12)


def test_delta_offset_is_64bit():
    # Llama-3-8B shape: 32 layers x 3 x 1024 x 4096 = 402,653,184 elements;
    # a single larger config overflows the reference's int.
    assert _lib.lib.glt_delta_offset(31, 2, 1024, 4096) == bx.delta_offset(31, 2, 1024, 4096)
    assert _lib.lib.glt_delta_offset(100, 2, 8192, 8192) == bx.delta_offset(100, 2, 8192, 8192)
    assert _lib.lib.glt_delta_offset(100, 2, 8192, 8192) > 2 ** 31


def test_model_create_reports_errors_without_throwing():
    c = G.default_config()
    h = C.c_void_p()
    st = _lib.lib.glt_model_create(C.byref(c.to_c()), 16, 512, 7, C.byref(h))
    assert st == 1 and "unknown model kind" in _lib.last_error()


def test_profile_kinds_match_header():
    # glt_model_profile_read writes GLT_PROF_KINDS entries into each buffer;
    # the Python mirror must size them the same or the call overruns them.
    text = open(HEADER).read()
    kinds = int(re.search(r"#define GLT_PROF_KINDS (\d+)", text).group(1))
    assert G.PROF_KINDS == kinds
    idx = {int(v): k.lower() for k, v in re.findall(r"#define GLT_PROF_(\w+) (\d+)", text) if k != "KINDS"}
    assert len(idx) == kinds
    assert idx[0] == "gate_up_fwd" and idx[12] == "attn_bwd" and idx[16] == "ce"


def test_gemm_pair_mode_switch_is_host_only():
    """glt_gemm_pair_mode sets and queries the process-wide GEMM tile mode
    without touching a device (mode -1 queries; other values are ignored)."""
    lib = _lib.lib
    prev = lib.glt_gemm_pair_mode(-1)
    assert prev in (0, 1)
    try:
        assert lib.glt_gemm_pair_mode(0) == 0
        assert lib.glt_gemm_pair_mode(-1) == 0
        assert lib.glt_gemm_pair_mode(7) == 0        # not a mode: query only
        assert lib.glt_gemm_pair_mode(1) == 1
        assert lib.glt_gemm_pair_mode(-1) == 1
    finally:
        lib.glt_gemm_pair_mode(prev)
    assert lib.glt_gemm_pair_mode(-1) == prev
