"""Resuming from the training state (glt_model_save/load_train_state): a
model that loads the state saved after k steps holds the saving model's fp32
graft and Adam moments bit for bit, its bf16 graft copies are refreshed, and
its next step matches the uninterrupted run's to the rounding of the fp32
atomics (split-K weight grads, dQ reduction)."""
import ctypes as C

import pytest
import torch

from glt_b200._lib import GltError, check, lib
from tests.test_gpu_decoder import gpu_model, problem, small_cfg

pytestmark = pytest.mark.gpu


def save_state(m, path, step, session=b"sess", domain=0):
    check(lib.glt_model_save_train_state(m.handle, path.encode(), session, domain, step))


def load_state(m, path, session=b"sess", domain=0):
    step = C.c_int64(-1)
    check(lib.glt_model_load_train_state(m.handle, path.encode(), session, domain, C.byref(step)))
    return step.value


@pytest.mark.parametrize("layout", ["concat", "overlay"])
def test_resume_continues_the_run(tmp_path, layout):
    over = dict(lr_peak=5e-3, lr_warmup_steps=1)
    if layout == "overlay":
        over.update(layout="overlay", max_domains=4, domain_id=0, slice_dim=160)
    rc = small_cfg(**over)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    a = gpu_model(rc, w, delta, B, T)
    for s in range(2):
        a.train_step(ids.cuda(), ood.cuda(), s, 6)
    p = str(tmp_path / "run.state")
    save_state(a, p, 2)
    b = gpu_model(rc, w, torch.zeros_like(delta), B, T)   # a different graft before the load
    assert load_state(b, p) == 2
    for which in ("weight", "adam_m", "adam_v"):
        assert torch.equal(a.read_graft(which), b.read_graft(which)), which
    # the loaded graft is live: base and grafted forwards of b match a's
    la = a.forward(ids.cuda())
    lb = b.forward(ids.cuda())
    assert torch.equal(la, lb)
    sa = a.train_step(ids.cuda(), ood.cuda(), 2, 6)
    sb = b.train_step(ids.cuda(), ood.cuda(), 2, 6)
    assert sb["total_loss"] == pytest.approx(sa["total_loss"], rel=1e-5)
    assert sb["lr"] == sa["lr"]
    torch.testing.assert_close(b.read_graft("weight"), a.read_graft("weight"), rtol=0, atol=1e-6)
    torch.testing.assert_close(b.read_graft("adam_v"), a.read_graft("adam_v"), rtol=1e-4, atol=1e-12)
    a.close()
    b.close()


def test_resume_refuses_other_domain_and_baked_model(tmp_path):
    rc = small_cfg()
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    a = gpu_model(rc, w, delta, B, T)
    p = str(tmp_path / "run.state")
    save_state(a, p, 0)
    before = a.read_graft("weight")
    with pytest.raises(GltError):
        load_state(a, p, domain=1)
    assert torch.equal(a.read_graft("weight"), before)
    a.shadow_bake()
    with pytest.raises(GltError):
        load_state(a, p)
    a.close()


def test_pipelined_steps_report_the_same_stats():
    """Steps enqueued without waiting (stats read one step behind through
    glt_model_step_stats) train exactly like steps that wait for their stats;
    only the last two steps' stats are kept."""
    rc = small_cfg(lr_peak=5e-3, lr_warmup_steps=1)
    B, T = 2, 128
    w, delta, ids, ood = problem(rc, B, T)
    a = gpu_model(rc, w, delta, B, T)
    sync = [a.train_step(ids, ood, s, 5) for s in range(5)]
    b = gpu_model(rc, w, delta, B, T)
    piped = []
    for s in range(5):
        assert b.train_step(ids, ood, s, 5, want_stats=False) is None   # host ids reused right away
        if s:
            piped.append(b.step_stats(s - 1))
    piped.append(b.step_stats(4))
    assert b.step_stats(3)["lr"] == sync[3]["lr"]
    with pytest.raises(GltError):
        b.step_stats(2)                      # no longer kept
    for x, y in zip(sync, piped):
        assert y["lr"] == x["lr"]
        for k in ("lm_loss", "silence_loss", "total_loss", "grad_norm"):
            assert y[k] == pytest.approx(x[k], rel=1e-4, abs=1e-7), k
    torch.testing.assert_close(b.read_graft("weight"), a.read_graft("weight"), rtol=0, atol=1e-5)
    a.close()
    b.close()
