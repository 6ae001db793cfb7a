"""graft_train end to end on the GPU, in the reference's certify sequence
(deploy/certify.sh): train a graft from safetensors base weights and .bin
token files, then --eval-only base (twice: the reload gate compares hashes),
--eval-only with the checkpoint (explicit graft) and --shadow-eval (baked).
The first logged step is checked against the fp32 oracle on the same batch
walk; the checkpoint against the oracle's GRFT parser."""
import csv
import os

import numpy as np
import pytest
import torch

from oracle import bitexact as bx
from oracle import ref_math as rm
from tests.cli_util import CLI, hf_tensors, key_values, run_cli, write_bin, write_safetensors
from tests.parity import make_decoder_weights

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not os.path.exists(CLI), reason="graft_train not built")]

DIMS = ["--hidden-dim", 256, "--intermediate-dim", 640, "--slice-dim", 160, "--vocab-size", 512,
        "--num-layers", 2, "--num-heads", 4, "--num-kv-heads", 2, "--rope-theta", 10000,
        "--graft-layer-start", 0, "--graft-layer-end", 1, "--domain-id", 1, "--max-domains", 4]


def oracle_cfg(**over):
    kw = dict(hidden_dim=256, intermediate_dim=640, slice_dim=160, vocab_size=512, num_layers=2,
              num_heads=4, num_kv_heads=2, rope_theta=10000.0, graft_layer_start=0, graft_layer_end=1,
              domain_id=1, max_domains=4, layout="overlay", graft_proj_gate=0, graft_proj_up=0,
              graft_proj_down=1, tie_embeddings=True)
    kw.update(over)
    return rm.GraftConfig(**kw).finalize()


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("cli")
    rc = oracle_cfg()
    w = make_decoder_weights(rc, seed=3, std=0.05)
    tensors = hf_tensors(w, tied=True)
    # norms stored as F32 and one projection as F16 exercise the dtype conversion
    dt = {"model.norm.weight": "F32", "model.layers.0.input_layernorm.weight": "F32",
          "model.layers.1.mlp.up_proj.weight": "F16"}
    write_safetensors(str(d / "model.safetensors"), tensors, dt)
    g = np.random.default_rng(11)
    T = 128
    dom = g.integers(0, 256, (6, T), dtype=np.int32)        # low half of the vocab
    ood1 = g.integers(256, 512, (3, T), dtype=np.int32)     # high half
    ood2 = g.integers(256, 512, (2, T), dtype=np.int32)
    ev = g.integers(0, 256, (5, T), dtype=np.int32)
    for name, arr in (("dom", dom), ("ood1", ood1), ("ood2", ood2), ("eval", ev)):
        write_bin(str(d / f"{name}.bin"), arr)
    # F16-stored weights round through fp16 before the model's bf16
    w["layers"][1]["wu"] = torch.from_numpy(
        bx.round_bf16(w["layers"][1]["wu"].numpy().astype(np.float16).astype(np.float32)).copy())
    return d, rc, w, dom, np.concatenate([ood1, ood2]), ev


def test_train_then_certify_sequence(files):
    d, rc, w, dom, ood, ev = files
    out = d / "run" / "ck.graft"
    out.parent.mkdir()
    r = run_cli("--safetensors", d / "model.safetensors", "--domain-data", d / "dom.bin",
                "--ood-data", d / "ood1.bin", d / "ood2.bin", "--output", out, "--steps", 3,
                "--batch-size", 2, "--lr", 1e-3, "--warmup-steps", 1, "--seed", 7,
                "--session-id", "s1", "--profile-graft-gemms", *DIMS)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    kv = key_values(r.stdout)
    assert int(kv["timed_steps"]) == 2 and kv["warmup_steps_excluded"] == "1"
    assert float(kv["sec_per_step_p50"]) > 0 and int(kv["peak_train_vram_mb"]) > 0
    rows = list(csv.DictReader(open(d / "run" / "ck_log.csv")))
    assert len(rows) == 3 and list(rows[0].keys())[-1] == "step_time_sec"
    assert float(rows[0]["grad_norm"]) == -1.0 and float(rows[1]["grad_norm"]) >= rc.gradient_clip_norm
    assert os.path.exists(d / "run" / "ck.graft_gemm_stats.json")
    # step 0 against the oracle on the same batch walk, graft zero-initialised
    dp, op = bx.batch_walk_start(7, dom.shape[0], ood.shape[0])
    ids, mask, _, _ = bx.batch_step(dom.reshape(-1), dom.shape[0], ood.reshape(-1), ood.shape[0],
                                    128, 2, dp, op)
    ids_t = torch.from_numpy(ids).view(2, 128)
    ood_t = torch.from_numpy(mask).view(2, 128)
    delta = torch.zeros(rc.total_projections * rc.slice_dim * rc.h_slice_dim)
    _, stats, _ = rm.compute_grads(ids_t, ood_t, w, delta, rc)
    assert float(rows[0]["lm_loss"]) == pytest.approx(stats["lm_loss"], rel=1e-2)
    # checkpoint: GRFT v4 with the reference metadata
    n, S, H = rc.total_projections, rc.slice_dim, rc.h_slice_dim
    buf = open(out, "rb").read()
    assert buf[:4] == b"GRFT"
    graft = bx.parse_grft(buf, 1, "s1", n, S, H)
    SH = S * H
    for l in range(rc.num_layers):  # contract-only: gate/up stay zero, down trained
        assert np.all(graft[(3 * l) * SH:(3 * l + 2) * SH] == 0)
        assert np.abs(graft[(3 * l + 2) * SH:(3 * l + 3) * SH]).max() > 0

    base_args = ["--safetensors", d / "model.safetensors", "--eval-data", d / "eval.bin",
                 "--batch-size", 2, "--session-id", "s1", *DIMS]
    a = run_cli("--eval-only", *base_args)
    a2 = run_cli("--eval-only", *base_args)
    b = run_cli("--eval-only", "--checkpoint", out, *base_args)
    c = run_cli("--shadow-eval", "--checkpoint", out, *base_args)
    for p in (a, a2, b, c):
        assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    A, A2, B, C = (key_values(p.stdout) for p in (a, a2, b, c))
    assert A["mode"] == "base" and B["mode"] == "grafted" and C["mode"] == "shadow"
    assert int(A["tokens"]) == ev.shape[0] * (ev.shape[1] - 1)
    # G3: a fresh base eval reproduces the first bit for bit
    assert A["logits_hash"] == A2["logits_hash"] and A["mean_ce"] == A2["mean_ce"]
    # the trained graft changes the logits; G2: baked == explicit within the bake budget
    assert B["logits_hash"] != A["logits_hash"]
    assert abs(float(C["mean_ce"]) - float(B["mean_ce"])) < 0.02
    assert C["shadow_baked"] == "true" and C["graft_freed_before_forward"] == "true"
    assert "graft forward calls=0" in c.stdout and "graft forward calls=0" in a.stdout
    # the base eval against the fp32 oracle
    logits, _, _, _ = rm.model_forward(torch.from_numpy(ev), w, None, rc)
    ce = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, rc.vocab_size),
                                           torch.from_numpy(ev)[:, 1:].reshape(-1).long())
    assert float(A["mean_ce"]) == pytest.approx(float(ce), rel=5e-3)


def test_checkpoint_domain_mismatch_is_refused(files):
    d, rc, w, dom, ood, ev = files
    out = d / "ck2.graft"
    r = run_cli("--safetensors", d / "model.safetensors", "--domain-data", d / "dom.bin",
                "--ood-data", d / "ood1.bin", "--output", out, "--steps", 1, "--batch-size", 2, *DIMS)
    assert r.returncode == 0, r.stderr[-2000:]
    dims = list(DIMS)
    dims[dims.index("--domain-id") + 1] = 2
    e = run_cli("--eval-only", "--checkpoint", out, "--safetensors", d / "model.safetensors",
                "--eval-data", d / "eval.bin", "--batch-size", 2, *dims)
    assert e.returncode != 0 and "domain" in e.stderr.lower()


def test_untied_transposed_lm_head_and_contract_probe(files, tmp_path):
    d, rc, w, dom, ood, ev = files
    # an untied copy whose lm_head is stored [D, V]: loaded transposed, same logits
    t = hf_tensors(w, tied=True)
    t["lm_head.weight"] = np.ascontiguousarray(w["embed"].numpy().T)
    write_safetensors(str(tmp_path / "untied.safetensors"), t)
    args = ["--eval-data", d / "eval.bin", "--batch-size", 2, *DIMS]
    a = run_cli("--eval-only", "--safetensors", d / "model.safetensors", *args)
    u = run_cli("--eval-only", "--safetensors", tmp_path / "untied.safetensors", *args)
    assert a.returncode == 0 and u.returncode == 0, u.stderr[-2000:]
    assert key_values(a.stdout)["logits_hash"] == key_values(u.stdout)["logits_hash"]
    # --contract-probe (graft_ops_impl.inc:158-212): out[0,11]=14, out[1,23]=65
    p = run_cli("--contract-probe", "--safetensors", d / "model.safetensors", "--domain-data",
                d / "dom.bin", "--ood-data", d / "ood1.bin", "--output", tmp_path / "p.graft",
                "--batch-size", 2, *DIMS)
    assert p.returncode == 0, p.stderr[-2000:]
    assert "out[0,11]=14" in p.stdout and "out[1,23]=65" in p.stdout
    assert "max_abs=65" in p.stdout


def test_stop_and_resume_continue_the_run(files, tmp_path):
    """--stop-after 2 + --save-state, then --resume-state, follows the same
    4-step schedule as one uninterrupted run: same batch walk, LR, losses
    (to the rounding of fp32 atomics) and trained graft; the resumed run
    appends to the log."""
    d, rc, w, dom, ood, ev = files
    common = ["--safetensors", d / "model.safetensors", "--domain-data", d / "dom.bin", "--ood-data",
              d / "ood1.bin", d / "ood2.bin", "--steps", 4, "--batch-size", 2, "--lr", 1e-3,
              "--warmup-steps", 1, "--seed", 7, "--session-id", "s1", *DIMS]
    full = run_cli(*common, "--output", tmp_path / "full.graft")
    part = run_cli(*common, "--output", tmp_path / "part.graft", "--stop-after", 2,
                   "--save-state", tmp_path / "s.state")
    rest = run_cli(*common, "--output", tmp_path / "part.graft", "--resume-state", tmp_path / "s.state",
                   "--save-state", tmp_path / "s2.state")
    for p in (full, part, rest):
        assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert "Resuming training at step 2 of 4" in rest.stdout
    a = list(csv.DictReader(open(tmp_path / "full_log.csv")))
    b = list(csv.DictReader(open(tmp_path / "part_log.csv")))
    assert [r["step"] for r in b] == ["0", "1", "2", "3"]
    for ra, rb in zip(a, b):
        assert float(rb["lr"]) == float(ra["lr"])
        for k in ("lm_loss", "silence_loss", "total_loss"):
            assert float(rb[k]) == pytest.approx(float(ra[k]), rel=1e-4, abs=1e-7), (ra["step"], k)
    blob = open(tmp_path / "s2.state", "rb").read()
    assert blob[:4] == b"GLTS" and b'"step":"4"' in blob
    n, S, H = rc.total_projections, rc.slice_dim, rc.h_slice_dim
    ga = bx.parse_grft(open(tmp_path / "full.graft", "rb").read(), 1, "s1", n, S, H)
    gb = bx.parse_grft(open(tmp_path / "part.graft", "rb").read(), 1, "s1", n, S, H)
    np.testing.assert_allclose(gb, ga, rtol=0, atol=1e-2 * float(np.abs(ga).max()))
