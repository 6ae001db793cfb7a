"""Data-parallel host logic on CPU (world size 2, gloo).

The GPU path all-reduces (sums) each layer's graft gradients over NCCL and
folds 1/world into the clip scale before AdamW.  This test runs the same
reduction with two gloo ranks over the fp32 oracle: each rank computes the
grads of its own microbatch, sums them with all_reduce, and the resulting
replicated update must equal the update from the mean of both ranks' grads
computed in one process; it also checks the max-over-ranks timing reduction
that bench.py uses."""
import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ref_math as rm


def _cfg():
    return rm.GraftConfig(hidden_dim=32, intermediate_dim=48, slice_dim=16, vocab_size=40,
                          num_layers=1, num_heads=4, num_kv_heads=2, graft_layer_start=0,
                          graft_layer_end=0, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                          layout="concat", lambda_silence=5.0, gradient_clip_norm=0.05).finalize()


def _problem(rank):
    cfg = _cfg()
    w = rm.init_weights(cfg, seed=0, std=0.2)
    g = torch.Generator().manual_seed(0)
    delta = torch.randn(cfg.total_projections * cfg.slice_dim * cfg.h_slice_dim, generator=g) * 0.2
    g2 = torch.Generator().manual_seed(100 + rank)
    ids = torch.randint(0, cfg.vocab_size, (2, 8), generator=g2, dtype=torch.int32)
    ood = torch.tensor([[0] * 8, [1] * 8], dtype=torch.int32)
    return cfg, w, delta, ids, ood


def _update_from_mean_grad(cfg, delta, gsum, world):
    g = gsum / world
    rm.clip_grads(g, cfg.gradient_clip_norm)
    out = delta.clone()
    rm.adamw(out, g, torch.zeros_like(out), torch.zeros_like(out), 0, 1e-3, cfg)
    return out


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w, delta, ids, ood = _problem(rank)
        grad, _, _ = rm.compute_grads(ids, ood, w, delta.clone(), cfg)
        dist.all_reduce(grad, op=dist.ReduceOp.SUM)
        upd = _update_from_mean_grad(cfg, delta, grad, world)
        t = torch.tensor([0.1 * (rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, upd, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_two_rank_graft_grad_allreduce_matches_mean():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort(key=lambda x: x[0])
    # replicas end identical and equal the single-process mean-gradient update
    torch.testing.assert_close(res[0][1], res[1][1], rtol=0, atol=0)
    gsum = None
    for r in range(world):
        cfg, w, delta, ids, ood = _problem(r)
        g, _, _ = rm.compute_grads(ids, ood, w, delta.clone(), cfg)
        gsum = g if gsum is None else gsum + g
    ref = _update_from_mean_grad(cfg, delta, gsum, world)
    torch.testing.assert_close(res[0][1], ref, rtol=1e-6, atol=1e-9)
    assert res[0][2] == pytest.approx(0.2) and res[1][2] == pytest.approx(0.2)


def _monitor_worker(rank, world, port, mode, q):
    """Rank 1 finishes steps 0 and 1, then leaves (posting its leave marker)
    or goes silent (a crash); rank 0 keeps stepping and must learn of it
    before it would start step 3's collectives."""
    import time
    from torch.distributed import TCPStore

    from glt_b200.graft import PeerLost, PeerMonitor
    store = TCPStore("127.0.0.1", port, world, is_master=(rank == 0), timeout=datetime.timedelta(seconds=30))
    mon = PeerMonitor(store, rank, world, timeout_s=1.0)
    last_done = -1
    try:
        for step in range(6):
            if step > 0:
                mon.wait_peers(step - 1)          # every peer finished the previous step
            if rank == 1 and step == 2:
                if mode == "leave":
                    mon.leave()
                q.put((rank, "stopped", step, None))
                return
            time.sleep(0.02)                      # the step's work
            mon.beat(step)
            last_done = step
        q.put((rank, "finished", last_done, None))
    except PeerLost as e:
        q.put((rank, "peer_lost", last_done, (e.peer, e.last_step, e.wanted, e.left)))
    finally:
        if rank == 0:
            time.sleep(0.5)                       # the store outlives its client


@pytest.mark.parametrize("mode", ["leave", "silent"])
def test_peer_monitor_detects_a_rank_that_leaves(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31500 + (os.getpid() % 2000) + (0 if mode == "leave" else 1)
    procs = [ctx.Process(target=_monitor_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r[0]: r for r in (q.get(timeout=60) for _ in range(world))}
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert res[1][1] == "stopped"
    kind, last_done, info = res[0][1], res[0][2], res[0][3]
    assert kind == "peer_lost"
    assert last_done == 2                          # rank 0 finished step 2, then stopped before step 3
    assert info == (1, 1, 2, mode == "leave")      # rank 1 last finished step 1; step 2 was awaited
