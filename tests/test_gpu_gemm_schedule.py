"""GEMM tile schedules (GLT_GEMM_SCHEDULE, read at glt_model_create): the
default round-robin units and dynamic claiming from a device counter give
the same results -- the same tiles, computed the same way, only on other
CTAs -- over several steps in a row (each launch re-arms the counter for
the next one on the stream)."""
import os

import pytest
import torch

from tests.test_gpu_decoder import gpu_model, problem, small_cfg
from tests.parity import assert_close_bf16

pytestmark = pytest.mark.gpu


def run(schedule, rc, w, delta, ids, ood, B, T):
    old = os.environ.get("GLT_GEMM_SCHEDULE")
    os.environ["GLT_GEMM_SCHEDULE"] = schedule
    try:
        m = gpu_model(rc, w, delta, B, T)
    finally:
        if old is None:
            del os.environ["GLT_GEMM_SCHEDULE"]
        else:
            os.environ["GLT_GEMM_SCHEDULE"] = old
    logits = [m.forward(ids.cuda()).clone()]
    losses = [m.train_step(ids.cuda(), ood.cuda(), s, 4)["total_loss"] for s in range(3)]
    logits.append(m.forward(ids.cuda()).clone())
    grad = m.read_graft("grad").cpu()
    m.close()
    return logits, losses, grad


@pytest.mark.parametrize("inter", [640, 1024])
def test_dynamic_claiming_matches_round_robin(inter):
    rc = small_cfg(intermediate_dim=inter, lr_peak=5e-3, lr_warmup_steps=1)
    B, T = 4, 128
    w, delta, ids, ood = problem(rc, B, T)
    ls, loss_s, g_s = run("static", rc, w, delta, ids, ood, B, T)
    ld, loss_d, g_d = run("dynamic", rc, w, delta, ids, ood, B, T)
    assert torch.equal(ls[0], ld[0])               # first forward: bit for bit
    for a, b in zip(loss_s, loss_d):
        assert b == pytest.approx(a, rel=1e-4)
    assert_close_bf16(ld[1].float(), ls[1].float(), "logits after 3 steps")
    assert_close_bf16(g_d, g_s, "graft grads of step 3")


def test_schedule_env_is_checked():
    from glt_b200._lib import GltError
    rc = small_cfg()
    w, delta, ids, ood = problem(rc, 2, 128)
    os.environ["GLT_GEMM_SCHEDULE"] = "sideways"
    try:
        with pytest.raises(GltError):
            gpu_model(rc, w, delta, 2, 128)
    finally:
        del os.environ["GLT_GEMM_SCHEDULE"]
