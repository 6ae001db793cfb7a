"""Grafted-MLP microbench sweep (hidden 4096, base intermediate 14336).

    python -m glt_b200.mlp_bench [--tokens 4096,16384,65536] [--slice 256,1024,4096]
                                 [--steps 5] [--warmup 3] [--mlp-store 0|1|auto]

One step = one grafted MLP block (RMSNorm -> [base | graft] gate/up GEMM with
fused SiLU*mul -> down GEMM, plus the backward to the graft weights and the
input, and the graft AdamW update) at hidden 4096, base intermediate 14336,
activations N(0,1), weights N(0,0.02).  Prints one JSON line per point with
the algorithmic TFLOP/s of the block, of its GEMMs, and per-kind kernel times.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

from . import graft as G


def run_point(M: int, S: int, steps: int, warmup: int, D: int = 4096, F: int = 14336,
              store: int = -1) -> dict:
    cfg = G.GraftConfig(hidden_dim=D, intermediate_dim=F, slice_dim=S, num_layers=1, num_heads=32,
                        num_kv_heads=8, vocab_size=0, layout=G.LAYOUT_CONCAT, graft_layer_start=0,
                        graft_layer_end=0, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                        allow_expansion_trap=1, adam_weight_decay=0.0, lambda_silence=0.0)
    m = G.GraftModel(cfg, 1, M, kind=G.MODEL_MLP_BLOCK)
    m.init_random(seed=5, std=0.02, graft_std=0.02, graft_down_std=0.02)
    if store >= 0:
        m.mlp_store(store)
    g = torch.Generator(device="cuda").manual_seed(M + S)
    x = torch.randn(M, D, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.randn(M, D, device="cuda", generator=g)
    for i in range(warmup):
        m.block_step(x, y, 1e-4, i, outputs=False)
    torch.cuda.synchronize()
    m.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        m.block_step(x, y, 1e-4, warmup + i, outputs=False)
    e1.record()
    torch.cuda.synchronize()
    m.profile(False)
    kms, kn = m.profile_read()
    store_on, _ = m.mlp_store()
    m.close()
    ms = e0.elapsed_time(e1) / steps
    Fp = F + S
    alg = M * (12.0 * D * Fp + 6.0 * D * S)   # fwd 6DF' + input grad 6DF' + graft dW 6DS
    gemm_kinds = [0, 1, 2, 6, 7, 8, 9, 10]   # the recompute kind (7) is zero with the MLP store
    gemm_ms = sum(kms[k] for k in gemm_kinds) / steps
    kernels = {G.PROF_NAMES[k]: round(kms[k] / steps, 4) for k in gemm_kinds}
    return {"tokens": M, "slice": S, "hidden": D, "ffn": F, "ms_per_step": ms,
            "block_tflops": alg / (ms / 1e3) / 1e12,
            "gemm_tflops_algorithmic": alg / (gemm_ms / 1e3) / 1e12,
            "gemm_tflops_executed": (alg + M * ((0.0 if store_on else 4.0 * D * Fp) + 2.0 * D * S))
                                    / (gemm_ms / 1e3) / 1e12,
            "mlp_activations": "stored" if store_on else "recomputed",
            "gemm_ms": gemm_ms, "non_gemm_ms": ms - gemm_ms, "kernel_ms": kernels}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="4096,16384,65536")
    ap.add_argument("--slice", default="256,1024,4096")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--mlp-store", choices=["0", "1", "auto"], default="auto",
                    help="1: the forward stores gate_pre/up for the backward; 0: the backward "
                         "recomputes them; auto: as the library decides")
    a = ap.parse_args(argv)
    store = -1 if a.mlp_store == "auto" else int(a.mlp_store)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    for S in [int(s) for s in a.slice.split(",")]:
        for M in [int(t) for t in a.tokens.split(",")]:
            print(json.dumps(run_point(M, S, a.steps, a.warmup, store=store)), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
