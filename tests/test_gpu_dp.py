"""Data-parallel training step on two GPUs against one-process training.

tests/dp_gpu_worker.py runs one step on each of two ranks joined by the
library's NCCL communicator (glt_dp_init): the graft-gradient all-reduce in
layer buckets during the backward (csrc/dp.cu), then the clip with 1/world
folded into its scale and AdamW on every rank.  The parent then checks:

* each rank's gradient buffer holds the sum of the two microbatches'
  gradients, each computed here by a one-GPU step on the same weights;
* the replicas' updated grafts are bit-identical;
* that update is the oracle's clip + AdamW (src/kernels_optimizer_impl.inc:
  11-77, grafting.hip:1150-1164) applied to the mean gradient, and the
  reported gradient norm is the mean gradient's norm.

Skipped when fewer than two GPUs are visible.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

from oracle import ref_math as rm
from tests.dp_gpu_worker import dp_problem, rank_batch
from tests.parity import load_weights, to_glt_config

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def single_gpu_grad(rc, w, delta, rank):
    from glt_b200 import graft as G
    ids, ood = rank_batch(rc, rank)
    m = G.GraftModel(to_glt_config(rc), 2, 128)
    try:
        load_weights(m, w)
        m.write_graft("weight", delta)
        m.train_step(ids, ood, step=0, total_steps=10)
        return m.read_graft("grad").cpu()
    finally:
        m.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_step_matches_single_process_mean_update(tmp_path):
    world = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "dp_gpu_worker.py"), str(tmp_path)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-4000:] + p.stderr[-4000:]
    ranks = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]

    rc, w, delta = dp_problem()
    for r in range(world):
        ids, _ = rank_batch(rc, r)
        assert torch.equal(ranks[r]["ids"], ids)
    g_sum = sum(single_gpu_grad(rc, w, delta, r) for r in range(world))
    scale = float(g_sum.abs().max())
    for r in range(world):
        # split-K weight grads and the attention dQ reduction use fp32
        # atomics, so separate runs agree to rounding, not bit for bit
        torch.testing.assert_close(ranks[r]["grad"], g_sum, rtol=1e-4, atol=1e-5 * scale)
    assert torch.equal(ranks[0]["grad"], ranks[1]["grad"]), "all-reduced gradients differ between ranks"
    assert torch.equal(ranks[0]["weight"], ranks[1]["weight"]), "replicas diverged after AdamW"

    g_mean = ranks[0]["grad"] / world
    norm = (float(g_mean.double().pow(2).sum()) + 1e-8) ** 0.5
    assert ranks[0]["stats"]["grad_norm"] == pytest.approx(norm, rel=1e-4)
    w_ref = delta.clone()
    g = g_mean.clone()
    rm.clip_grads(g, rc.gradient_clip_norm)
    rm.adamw(w_ref, g, torch.zeros_like(w_ref), torch.zeros_like(w_ref), 0, rc.get_lr(0, 10), rc)
    torch.testing.assert_close(ranks[0]["weight"], w_ref, rtol=1e-5, atol=1e-8)
    # after glt_dp_abort each rank trains alone: its next gradient is its own
    for r in range(world):
        assert ranks[r]["async_error"] == 0
        assert ranks[r]["solo_stats"]["total_loss"] > 0
        assert not torch.equal(ranks[r]["solo_grad"], ranks[0]["grad"])
    assert not torch.equal(ranks[0]["solo_grad"], ranks[1]["solo_grad"])
