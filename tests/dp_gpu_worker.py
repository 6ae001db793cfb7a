"""One rank of the data-parallel GPU check in tests/test_gpu_dp.py.

Launched by torch.distributed.run with one process per GPU.  Every rank
builds the same grafted decoder (same base and graft weights), takes its own
microbatch (seed 500 + rank), joins the library's NCCL communicator
(glt_dp_init; the unique id travels over a gloo group) and runs one training
step: the graft gradients are all-reduced in layer buckets during the
backward, then clip and AdamW run on every rank.  It saves its ids, the
summed gradients, the updated graft and the step statistics to
<out_dir>/rank<r>.pt for the parent test to check; then, with no
collective in flight, it aborts the communicator (glt_dp_abort, the path of
a rank whose peer has left) and runs one more step on its own GPU.

    python -m torch.distributed.run --nproc-per-node 2 tests/dp_gpu_worker.py OUT_DIR
"""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def dp_problem():
    """Same decoder for every rank: 5 layers, so the default 4-layer gradient
    buckets end with a partial one ([4, 5) then [0, 4))."""
    from oracle import ref_math as rm
    from tests.parity import make_decoder_weights
    rc = rm.GraftConfig(hidden_dim=256, intermediate_dim=640, slice_dim=128, vocab_size=512,
                        num_layers=5, num_heads=4, num_kv_heads=2, rope_theta=10000.0,
                        graft_layer_start=0, graft_layer_end=4, graft_proj_gate=1, graft_proj_up=1,
                        graft_proj_down=1, layout="concat", lambda_silence=5.0,
                        gradient_clip_norm=0.05).finalize()
    w = make_decoder_weights(rc, seed=21, std=0.05)
    g = torch.Generator().manual_seed(22)
    delta = torch.randn(rc.total_projections * rc.slice_dim * rc.h_slice_dim, generator=g) * 0.05
    return rc, w, delta


def rank_batch(rc, rank, B=2, T=128):
    g = torch.Generator().manual_seed(500 + rank)
    ids = torch.randint(0, rc.vocab_size, (B, T), generator=g, dtype=torch.int32)
    ood = torch.zeros(B, T, dtype=torch.int32)
    ood[B // 2:] = 1
    return ids, ood


def main():
    out_dir = sys.argv[1]
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from glt_b200 import graft as G
    from tests.parity import load_weights, to_glt_config
    rc, w, delta = dp_problem()
    ids, ood = rank_batch(rc, rank)
    m = G.GraftModel(to_glt_config(rc), 2, 128)
    load_weights(m, w)
    m.write_graft("weight", delta)
    uid = [G.GraftModel.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.dp_init(uid[0], rank, world)
    st = m.train_step(ids, ood, step=0, total_steps=10)
    torch.cuda.synchronize()
    out = dict(ids=ids, ood=ood, grad=m.read_graft("grad").cpu(), weight=m.read_graft("weight").cpu(),
               stats=st, async_error=m.dp_async_error())
    # between steps, no collective in flight: a rank that learned on the host
    # that a peer left aborts the communicator and carries on alone
    m.dp_abort()
    out["solo_stats"] = m.train_step(ids, ood, step=1, total_steps=10)
    out["solo_grad"] = m.read_graft("grad").cpu()
    m.dp_finalize()
    m.close()
    torch.save(out, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
