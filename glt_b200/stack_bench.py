"""Stacked-graft inference at the Llama-3-8B shape: four independently seeded
sibling grafts of width 512 active at once on the Llama-3-8B shape, prefill
forward of batch 8 x seq 4096 uniform-random tokens, explicit stack versus
the same grafts shadow-baked into the base MLP weights.

    python -m glt_b200.stack_bench [--geometry overlay|concat|both] [--batch 8] [--seq 4096]
                                   [--layers 32] [--steps 3] [--warmup 2]
    torchrun --nproc-per-node N ... python -m glt_b200.stack_bench   (replicas, one per GPU)

overlay: the reference's geometry -- domain d's graft at intermediate rows
  [512d, 512(d+1)) and hidden columns [1024d, 1024(d+1)) (max_domains 4),
  assembled by glt_stack_grafts into one block-diagonal graft.
concat:  the four slices side by side, [base | s0 | s1 | s2 | s3].

Under torchrun every rank holds the same base model and stack and runs its
own prefill batch (weak scaling, no collective on the data path); the only
exchange is one reduce of the metrics at the end.  Prints one JSON line per
geometry: prefill tokens/s of the stacked and of the baked forward (CUDA
events on the launching stream, whole forward including the LM head, max
over ranks, summed over ranks for the aggregate), and the logits agreement
over every logit (worst over the ranks) (max |stack - baked| / max |stack| and the
cosine), checked against the bf16 gate (<= 2e-2, >= 0.999), and the mean
next-token CE of both models over the batch against the reference's own bake
acceptance gate (|CE_shadow - CE_explicit| < 0.02).  Base weights are
random-init N(0, 0.02) (no checkpoint is available here).  Grafts are
N(0, --graft-std): the default 3e-4 gives a per-token graft energy (RMS of the
injected delta) of about sqrt(1024) * 3e-4 = 0.0096, the scale of the
reference's trained grafts (domain graft energy 0.0091 in its
runs/medical_all3.run.json); --graft-std 0.02 is a stress case in which each
graft is as large as the base weights it overlays.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import sys

import torch

from . import _lib
from . import graft as G

MAX_REL, MIN_COS = 2e-2, 0.999
EPS_CE_BAKE = 0.02   # the reference's certify gate G2 on |CE_shadow - CE_explicit| (deploy/config.sh:40)


def logits_agreement(a: torch.Tensor, b: torch.Tensor, chunk: int = 4096) -> tuple[float, float]:
    """max |a - b| / max |b| and cosine over all logits, chunked fp32 on the GPU."""
    dmax = torch.zeros((), device=a.device, dtype=torch.float64)
    bmax = torch.zeros_like(dmax)
    dot = torch.zeros_like(dmax)
    na = torch.zeros_like(dmax)
    nb = torch.zeros_like(dmax)
    for r in range(0, a.shape[0], chunk):
        x = a[r:r + chunk].float()
        y = b[r:r + chunk].float()
        dmax = torch.maximum(dmax, (x - y).abs().max().double())
        bmax = torch.maximum(bmax, y.abs().max().double())
        dot += (x.double() * y.double()).sum()
        na += x.double().pow(2).sum()
        nb += y.double().pow(2).sum()
    return float(dmax / bmax), float(dot / (na.sqrt() * nb.sqrt()))


def l2_rel(a: torch.Tensor, b: torch.Tensor, chunk: int = 4096) -> float:
    """||a - b|| / ||b|| over all logits."""
    num = torch.zeros((), device=a.device, dtype=torch.float64)
    den = torch.zeros_like(num)
    for r in range(0, a.shape[0], chunk):
        x = a[r:r + chunk].double()
        y = b[r:r + chunk].double()
        num += (x - y).pow(2).sum()
        den += y.pow(2).sum()
    return float((num / den).sqrt())


def run(geometry: str, a, world: int, rank: int, dist) -> dict:
    N, S_each, D, F, L = 4, 512, 4096, 14336, a.layers
    V, nh, nkv = 128256, 32, 8
    B, T = a.batch, a.seq
    common = dict(hidden_dim=D, intermediate_dim=F, vocab_size=V, num_layers=L, num_heads=nh,
                  num_kv_heads=nkv, head_dim=128, rope_theta=5e5, tie_embeddings=0, graft_layer_start=0,
                  graft_layer_end=L - 1, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                  allow_expansion_trap=1)
    H_each = D // N
    if geometry == "overlay":
        cfg = G.GraftConfig(slice_dim=N * S_each, max_domains=1, domain_id=0, layout=G.LAYOUT_OVERLAY,
                            **common)
    else:
        cfg = G.GraftConfig(slice_dim=N * S_each, max_domains=4, domain_id=0, layout=G.LAYOUT_CONCAT,
                            **common)
    m = G.GraftModel(cfg, B, T, kind=G.MODEL_DECODER)
    # replicas: the same base weights and grafts on every rank, each rank its own prefill batch
    m.init_random(seed=1234, std=0.02, graft_std=0.0, graft_down_std=0.0)
    stream = torch.cuda.current_stream()
    gen = [torch.Generator(device="cuda").manual_seed(100 + d) for d in range(N)]
    if geometry == "overlay":
        sib = [torch.randn(3 * L * S_each * H_each, device="cuda", generator=gen[d]) * a.graft_std
               for d in range(N)]
        graft = torch.empty(3 * L * N * S_each * N * H_each, device="cuda")
        ptrs = (C.c_void_p * N)(*[t.data_ptr() for t in sib])
        _lib.check(_lib.lib.glt_stack_grafts(ptrs, N, L, S_each, H_each, C.c_void_p(graft.data_ptr()),
                                             C.c_void_p(stream.cuda_stream)))
        del sib
    else:
        parts = [torch.randn(3 * L, S_each, D, device="cuda", generator=gen[d]) * a.graft_std
                 for d in range(N)]
        graft = torch.cat(parts, dim=1).reshape(-1)
        del parts
    m.write_graft("weight", graft)
    del graft
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    ids = torch.randint(0, V, (B, T), device="cuda", generator=g, dtype=torch.int32)
    logits_stack = torch.empty(B * T, V, dtype=torch.bfloat16, device="cuda")
    logits_baked = torch.empty_like(logits_stack)

    def fwd(use_graft: bool, out: torch.Tensor):
        _lib.check(_lib.lib.glt_forward(m.handle, C.c_void_p(ids.data_ptr()), 0, int(use_graft),
                                        C.c_void_p(out.data_ptr()), C.c_void_p(stream.cuda_stream)))

    def timed(use_graft: bool, out: torch.Tensor) -> float:
        for _ in range(a.warmup):
            fwd(use_graft, out)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            fwd(use_graft, out)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / a.steps
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
        return ms

    ms_stack = timed(True, logits_stack)
    ce_stack = m.eval(ids, use_graft=True)["mean_ce"]
    logits_base = torch.empty_like(logits_stack)
    fwd(False, logits_base)   # base model (graft columns skipped) for the graft's effect size
    m.shadow_bake()
    ms_baked = timed(False, logits_baked)
    ce_baked = m.eval(ids, use_graft=False)["mean_ce"]
    rel, cos = logits_agreement(logits_baked, logits_stack)
    l2 = l2_rel(logits_baked, logits_stack)
    effect = l2_rel(logits_base, logits_stack)
    del logits_base
    m.close()
    if dist:
        # the one exchange of the replicas: their metrics, reduced once at the end
        # (worst agreement over the ranks, mean CE over the ranks' batches)
        t = torch.tensor([rel, -cos, l2, effect, ce_stack, ce_baked], device="cuda", dtype=torch.float64)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        rel, cos, l2, effect = float(tmax[0]), -float(tmax[1]), float(tmax[2]), float(tmax[3])
        ce_stack, ce_baked = float(t[4]) / world, float(t[5]) / world
    tok = world * B * T
    return {"config": "stacked-graft inference, llama3-8b shape, 4 x 512 sibling grafts, prefill 8 x 4096", "geometry": geometry,
            "stack": f"{N} sibling grafts x {S_each}", "model": f"llama3-8b shape, {L} layers",
            "batch": B, "seq": T, "n_gpus": world, "parallelism": f"dp{world} (replicas, one metrics reduce)",
            "scaling": "weak", "dtype": "bf16", "data": "synthetic",
            "stack_ms": ms_stack, "stack_tokens_per_s": tok / (ms_stack / 1e3),
            "baked_ms": ms_baked, "baked_tokens_per_s": tok / (ms_baked / 1e3),
            "graft_std": a.graft_std, "logits_max_rel": rel, "logits_cos": cos, "logits_l2_rel": l2,
            "graft_effect_l2_rel": effect,
            "gate": {"max_rel": MAX_REL, "min_cos": MIN_COS, "pass": bool(rel <= MAX_REL and cos >= MIN_COS)},
            "mean_ce_stack": ce_stack, "mean_ce_baked": ce_baked,
            "bake_ce_gate": {"eps": EPS_CE_BAKE, "delta": abs(ce_baked - ce_stack),
                             "pass": bool(abs(ce_baked - ce_stack) < EPS_CE_BAKE)}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--geometry", choices=["overlay", "concat", "both"], default="both")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--graft-std", type=float, default=3e-4)
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    ok = True
    for geo in (["overlay", "concat"] if a.geometry == "both" else [a.geometry]):
        r = run(geo, a, world, rank, dist)
        ok = ok and r["gate"]["pass"]
        if rank == 0:
            print(json.dumps(r), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
