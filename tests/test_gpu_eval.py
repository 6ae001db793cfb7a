"""Eval-only / shadow-eval metrics (grafting.hip:446-713) through glt_model_eval:
the on-device CE, logits sum / L2 and the row-parallel FNV-1a fingerprint
against the same quantities computed on the host from the model's own bf16
logits (the reference's host loop), the CE against the fp32 oracle, run-to-run
determinism (the certify reload gate compares hashes), and the shadow-eval
sequence: bake, graft freed, base-only forward."""
import numpy as np
import pytest
import torch

from oracle import ref_math as rm
from oracle.bitexact import fnv1a64_f32
from tests.test_gpu_decoder import gpu_model, problem, small_cfg

pytestmark = pytest.mark.gpu


def host_metrics(m, ids, B, use_graft):
    """The reference's host loop over batches of B sequences, from glt_forward logits."""
    n, T = ids.shape
    V = m.cfg.vocab_size
    nll, tokens, s, sq = 0.0, 0, 0.0, 0.0
    all_logits = []
    for s0 in range(0, n, B):
        cur = min(B, n - s0)
        batch = ids[s0:s0 + cur]
        if cur < B:  # rows are independent: pad with copies, keep the first cur
            batch = torch.cat([batch, batch[:1].repeat(B - cur, 1)])
        lg = m.forward(batch.cuda(), use_graft=use_graft).float().cpu().view(B, T, V)[:cur]
        ce = torch.nn.functional.cross_entropy(lg[:, :-1].reshape(-1, V),
                                               ids[s0:s0 + cur, 1:].reshape(-1).long(),
                                               reduction="sum")
        nll += float(ce)
        tokens += cur * (T - 1)
        arr = lg.numpy().astype(np.float64)
        s += float(arr.sum())
        sq += float((arr * arr).sum())
        all_logits.append(lg.numpy())
    return dict(tokens=tokens, mean_ce=nll / tokens, logits_sum=s, logits_l2=sq ** 0.5,
                logits_hash=fnv1a64_f32(np.concatenate(all_logits)))


@pytest.mark.parametrize("use_graft", [True, False])
def test_eval_metrics_match_host_loop(use_graft):
    rc = small_cfg()
    B, T, n = 2, 128, 5          # batches of 2, 2 and a short last batch of 1
    w, delta, _, _ = problem(rc, B, T, graft_std=0.05)
    ids = torch.randint(0, rc.vocab_size, (n, T), generator=torch.Generator().manual_seed(7),
                        dtype=torch.int32)
    m = gpu_model(rc, w, delta, B, T)
    ev = m.eval(ids, use_graft=use_graft)
    want = host_metrics(m, ids, B, use_graft)
    m.close()
    assert ev["tokens"] == want["tokens"] == n * (T - 1)
    assert ev["logits_hash"] == want["logits_hash"]
    assert ev["logits_sum"] == pytest.approx(want["logits_sum"], rel=1e-9, abs=1e-6)
    assert ev["logits_l2"] == pytest.approx(want["logits_l2"], rel=1e-9)
    assert ev["mean_ce"] == pytest.approx(want["mean_ce"], rel=1e-5)
    assert ev["ppl"] == pytest.approx(np.exp(ev["mean_ce"]), rel=1e-12)
    assert ev["graft_forward_calls"] == (rc.num_layers * 3 if use_graft else 0)


def test_eval_ce_matches_fp32_oracle_and_is_deterministic():
    rc = small_cfg()
    B, T = 2, 128
    w, delta, ids, _ = problem(rc, B, T, graft_std=0.05)
    m = gpu_model(rc, w, delta, B, T)
    a = m.eval(ids)
    b = m.eval(ids.cuda())
    m.close()
    assert a == b  # bit-identical, host or device ids
    logits, _, _, _ = rm.model_forward(ids, w, delta, rc)
    ce = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, rc.vocab_size),
                                           ids[:, 1:].reshape(-1).long())
    assert a["mean_ce"] == pytest.approx(float(ce), rel=5e-3)


def test_shadow_eval_concat_equals_explicit_and_frees_graft():
    rc = small_cfg()
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T, graft_std=0.05)
    m = gpu_model(rc, w, delta, B, T)
    explicit = m.eval(ids, use_graft=True)
    base = m.eval(ids, use_graft=False)
    assert base["logits_hash"] != explicit["logits_hash"]
    m.shadow_bake()
    shadow = m.eval(ids, use_graft=False)
    # concat: the base has zero rows in the graft columns, so bf16(0 + delta)
    # is the explicit path's bf16 graft weight and the logits are identical
    assert shadow["logits_hash"] == explicit["logits_hash"]
    assert shadow["mean_ce"] == explicit["mean_ce"]
    assert shadow["graft_forward_calls"] == 0
    from glt_b200._lib import GltError
    with pytest.raises(GltError, match="twice"):
        m.shadow_bake()
    with pytest.raises(GltError, match="freed"):
        m.eval(ids, use_graft=True)
    with pytest.raises(GltError):
        m.train_step(ids, ood, step=0, total_steps=1)
    m.close()
