#!/usr/bin/env python
"""Graft-train throughput at the Llama-3-8B shape.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one full grafted training step of the decoder (embedding, 32
layers with attention and the [base | graft] SwiGLU MLP, LM head + CE on
domain tokens, OOD silence loss, backward -- SwiGLU's backward fused into the
dh GEMM from the gate_pre/up the forward stored, or the reference's FFN
recompute when the device has no room for them -- all-reduce of
the graft gradients across ranks, global-norm clip, graft-only AdamW) over a
16 x 2048-token microbatch per GPU.  Prints one JSON line (rank 0).

value  tokens/s of the whole job with the token ids already on the device
       (CUDA events on the step stream, max over ranks);
e2e    the same metric through glt_train_step with pinned-host inputs copied
       in and the step statistics read back every step;
roofline  the dominant kernel (the gate/up GEMM with fused SwiGLU) timed live
       with CUDA events around each of its launches, in a second pass of the
       same steps right after the timed region (the events cost ~0.3% of a
       step at this shape, so the timed region itself runs without them);
extra  the same step recomputing the FFN (recompute_ffn) instead of keeping
       the forward's gate_pre/up;
cpu_baseline  the fp32 CPU oracle on this host's cores, one decoder layer on
       a bounded token sample, extrapolated per token.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (layers, hidden, ffn, slice, heads, kv_heads, head_dim, vocab, theta, tie, batch, seq)
    "c3": dict(num_layers=32, hidden_dim=4096, intermediate_dim=14336, slice_dim=1024, num_heads=32,
               num_kv_heads=8, head_dim=128, vocab_size=128256, rope_theta=500000.0,
               tie_embeddings=0, batch=16, seq=2048,
               label="llama3-8b graft-train: 32L d4096 ffn14336 + graft 1024, "
                     "32q/8kv hd128, vocab 128256, 16x2048 tokens/GPU"),
    "c2": dict(num_layers=24, hidden_dim=896, intermediate_dim=4864, slice_dim=512, num_heads=14,
               num_kv_heads=2, head_dim=64, vocab_size=151936, rope_theta=1000000.0,
               tie_embeddings=1, batch=8, seq=1024,
               label="qwen2.5-0.5b graft-train: 24L d896 ffn4864 + graft 512, "
                     "14q/2kv hd64, vocab 151936, 8x1024 tokens/GPU"),
}
METRIC = "graft-train tokens/s at Llama-3-8B shape, 1-8 B200; MLP GEMM % of bf16 peak"
# ncu DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one
# gate/up GEMM launch at the config-3 layer shape (M = 32768 tokens, K = 4096,
# N = 2F' = 30720), captured on the identical launch of `python -m
# glt_b200.mlp_bench --tokens 32768 --slice 1024 [--mlp-store 0]` (the full
# training step is too large for a capture under the profiling rules), keyed
# by (CTA-pair GEMMs, MLP store); algorithmic bytes 3.54 GB with the store
# (x 268 MB + W_gu 252 MB read, h 1007 MB + bf16 gate_pre/up 2014 MB
# written), 1.53 GB without:
#   pairs, store on:      3,273,385,472 B read + 2,996,351,232 B written
#   pairs, recompute:     4,736,081,152 B read + 1,001,093,888 B written
#   one SM, store on:     2,496,413,184 B read + 2,991,854,080 B written
#   one SM, recompute:    2,329,381,376 B read +   996,020,480 B written
GATE_UP_TRAFFIC_BYTES = {(True, True): 3273385472 + 2996351232, (True, False): 4736081152 + 1001093888,
                         (False, True): 2496413184 + 2991854080, (False, False): 2329381376 + 996020480}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return dict(hbm=d["hbm_gbs"], tf=d["bf16_tflops"], tf_sus=d["bf16_tflops_sustained"],
                    src="measured")
    except Exception:  # noqa: BLE001
        return dict(hbm=6650.0, tf=1590.0, tf_sus=1400.0, src="fallback")


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set()
        for r in rows:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[k].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows),
                "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows),
                "samples": len(rows), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# CPU oracle baseline (bounded sample, extrapolated)
# ---------------------------------------------------------------------------
def cpu_oracle_sample(wl: dict, tokens: int, reps: int = 2):
    """Times one grafted decoder layer (forward + reference-structured backward)
    of the fp32 CPU oracle on `tokens` tokens; returns (seconds per layer pass, cores)."""
    import torch
    from oracle import ref_math as rm
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rc = rm.GraftConfig(hidden_dim=wl["hidden_dim"], intermediate_dim=wl["intermediate_dim"],
                        slice_dim=wl["slice_dim"], vocab_size=wl["vocab_size"], num_layers=1,
                        num_heads=wl["num_heads"], num_kv_heads=wl["num_kv_heads"],
                        head_dim=wl["head_dim"], rope_theta=wl["rope_theta"], graft_layer_start=0,
                        graft_layer_end=0, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                        layout="concat").finalize()
    g = torch.Generator().manual_seed(0)
    D, F = rc.hidden_dim, rc.intermediate_dim
    nh, nkv, hd = rc.num_heads, rc.num_kv_heads, rc.head_dim

    def rn(*s):
        return torch.randn(*s, generator=g) * 0.02

    lw = dict(in_norm=torch.ones(D), wq=rn(nh * hd, D), wk=rn(nkv * hd, D), wv=rn(nkv * hd, D),
              wo=rn(D, nh * hd), post_norm=torch.ones(D), wg=rn(F, D), wu=rn(F, D), wd=rn(D, F))
    delta = rn(3 * rc.slice_dim * rc.h_slice_dim)
    x = torch.randn(1, tokens, D, generator=g)
    ood = torch.zeros(tokens, dtype=torch.int32)
    ood[tokens // 2:] = 1
    times = []
    for i in range(reps + 1):
        t0 = time.perf_counter()
        y, saved = rm.layer_forward(x, lw, delta, rc, 0)
        grad = torch.zeros_like(delta)
        rm.layer_backward(torch.randn_like(y) * 1e-3, lw, delta, saved, rc, 0, ood, 1e-4, grad)
        dt = time.perf_counter() - t0
        if i:
            times.append(dt)
    return statistics.median(times), cores


def run_reference_arm(args, wl):
    """--impl reference: the reference's CPU path is the fp32 oracle port (the
    HIP/ROCm reference cannot be built here); each step is a bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    tokens = args.cpu_tokens
    per = []
    for i in range(args.warmup + args.steps):
        s, cores = cpu_oracle_sample(wl, tokens, reps=1)
        if i >= args.warmup:
            per.append(s)
    sec_layer = statistics.median(per)
    tok_s = tokens / (sec_layer * wl["num_layers"])
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": wl["batch"] * wl["seq"] / tok_s * 1e3,
        "extrapolated": True,
        "sample_ms_per_step": sec_layer * 1e3,
        "higher_is_better": True, "scaling": "none: one host's cores, the same line at every --gpus",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02) weights, N(0,1) activations",
        "config": {"workload": wl["label"], "global_batch": wl["batch"], "seq_len": wl["seq"],
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"fp32 CPU oracle: one grafted decoder layer forward+backward on "
                                   f"1x{tokens} tokens per step ({sec_layer * 1e3:.0f} ms measured), "
                                   f"extrapolated linearly to {wl['num_layers']} layers and "
                                   f"{wl['batch']}x{wl['seq']} tokens (LM head excluded); "
                                   f"ms_per_step is that extrapolation",
                         "sampled_layers": 1, "sampled_tokens": tokens, "extrapolated": True},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


NCCL_ALGOS = {0: "Tree", 1: "Ring", 2: "CollNetDirect", 3: "CollNetChain", 4: "NVLS", 5: "NVLSTree", 6: "PAT"}
NCCL_PROTOS = {0: "LL", 1: "LL128", 2: "Simple"}


def nccl_summary(path):
    """The algorithm/protocol NCCL chose for each all-reduce size (its TUNING
    lines, 'AllReduce: <bytes> Bytes -> Algo <a> proto <p> ...'), and the
    communicators it built."""
    import re
    try:
        text = open(path).read()
    except OSError:
        return {"log": "unavailable"}
    picks = {}
    # NCCL prints the algorithm and protocol by index (older releases) or by
    # name (2.2x: "Algo RING proto SIMPLE")
    def name(table, v):
        return table.get(int(v), v) if v.isdigit() else v

    for m in re.finditer(r"AllReduce: (\d+) Bytes -> Algo (\w+) proto (\w+)", text):
        key = f"{int(m.group(1))} B"
        picks.setdefault(key, {"algo": name(NCCL_ALGOS, m.group(2)),
                               "proto": name(NCCL_PROTOS, m.group(3)), "calls": 0})
        picks[key]["calls"] += 1
    nvls = [ln.split("NCCL INFO")[-1].strip() for ln in text.splitlines() if "NVLS" in ln][:4]
    tuning = [ln.split("NCCL INFO")[-1].strip() for ln in text.splitlines() if " Algo " in ln][:3]
    return {"allreduce": picks, "nvls_lines": nvls, "tuning_lines": tuning, "version": (re.findall(r"NCCL version [^\s]+", text) or [None])[0]}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c3")
    ap.add_argument("--cpu-tokens", type=int, default=512)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mlp-store", choices=["0", "1", "auto"], default="auto",
                    help="FFN pre-activations in the timed steps: 1 stored by the forward, "
                         "0 recomputed in the backward (recompute_ffn), auto as the library decides")
    ap.add_argument("--recompute-steps", type=int, default=None,
                    help="steps of the extra recompute-mode timing after the main one "
                         "(default: --steps; 0 skips it)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference_arm(args, wl)

    import torch
    from glt_b200 import _lib
    from glt_b200 import graft as G

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    nccl_log = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        if "NCCL_DEBUG_FILE" not in os.environ:
            # NCCL's own record of the algorithm and protocol it picks for each
            # all-reduce (TUNING lines), one file per rank, summarised in the line
            nccl_log = os.path.join("/tmp", f"glt_bench_nccl.{os.getpid()}.log")
            if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
                os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.update(NCCL_DEBUG_SUBSYS=os.environ.get("NCCL_DEBUG_SUBSYS", "INIT,TUNING"),
                              NCCL_DEBUG_FILE=nccl_log)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    B, T = wl["batch"], wl["seq"]
    cfg = G.GraftConfig(
        hidden_dim=wl["hidden_dim"], intermediate_dim=wl["intermediate_dim"], slice_dim=wl["slice_dim"],
        vocab_size=wl["vocab_size"], num_layers=wl["num_layers"], num_heads=wl["num_heads"],
        num_kv_heads=wl["num_kv_heads"], head_dim=wl["head_dim"], rope_theta=wl["rope_theta"],
        tie_embeddings=wl["tie_embeddings"], layout=G.LAYOUT_CONCAT, graft_layer_start=0,
        graft_layer_end=wl["num_layers"] - 1, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
        allow_expansion_trap=1, lambda_silence=5.0, lr_peak=2e-4, lr_warmup_steps=20)
    model = G.GraftModel(cfg, B, T)
    if args.mlp_store != "auto":
        model.mlp_store(int(args.mlp_store))
    # replicas start identical; graft down N(0,0.02) so no zero-skipping shortcut exists
    model.init_random(seed=1234, std=0.02, graft_std=0.02, graft_down_std=0.02)
    if world > 1:
        uid = [G.GraftModel.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.dp_init(uid[0], rank, world)

    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    ids = torch.randint(0, wl["vocab_size"], (B, T), device="cuda", dtype=torch.int32, generator=gen)
    ood = torch.zeros(B, T, dtype=torch.int32, device="cuda")
    ood[B // 2:] = 1
    total_steps = args.warmup + args.steps
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    step = 0
    for _ in range(args.warmup):
        model.train_step(ids, ood, step, total_steps, want_stats=False)
        step += 1
    barrier()
    smi_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            smi_index = int(vis.split(",")[local])
        except ValueError:
            pass
    launches0 = C.c_uint64()
    _lib.check(_lib.lib.glt_launch_count(C.byref(launches0)))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(smi_index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            model.train_step(ids, ood, step, total_steps, want_stats=False)
            step += 1
        e1.record(stream)
        torch.cuda.synchronize()
    launches1 = C.c_uint64()
    _lib.check(_lib.lib.glt_launch_count(C.byref(launches1)))
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    tokens_per_step = world * B * T

    # per-kind kernel times: the same steps again with CUDA events recorded on
    # the launching stream around every launch (kept out of the main region,
    # whose value they would lower by their own cost)
    _lib.check(_lib.lib.glt_model_profile(model.handle, 1))
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(args.steps):
        model.train_step(ids, ood, step, total_steps + args.steps, want_stats=False)
        step += 1
    p1.record(stream)
    torch.cuda.synchronize()
    _lib.check(_lib.lib.glt_model_profile(model.handle, 0))
    barrier()
    profiled_ms = max_over_ranks(p0.elapsed_time(p1) / args.steps)
    value = tokens_per_step / (ms / 1e3)
    kms, kn = model.profile_read(reset=True)   # sized by the library's GLT_PROF_KINDS
    M = B * T
    D, F, S, L = wl["hidden_dim"], wl["intermediate_dim"], wl["slice_dim"], wl["num_layers"]
    Fp = F + S
    gu_flops = 2.0 * M * D * 2 * Fp                      # one gate/up launch
    gu_ms = kms[0] / max(kn[0], 1)
    pk = peaks()
    achieved = gu_flops / (gu_ms / 1e3) / 1e12
    mlp_alg = (12.0 * D * Fp + 6.0 * D * S) * M * L      # per step, recompute excluded
    mlp_kinds = (0, 1, 2, 6, 7, 8, 9, 10)
    mlp_ms = sum(kms[k] for k in mlp_kinds) / args.steps
    store_on, store_bytes = model.mlp_store()
    mlp_exec = mlp_alg + (2.0 * D * S + (0.0 if store_on else 4.0 * D * Fp)) * M * L  # + delta_down (+ recompute)
    pair = _lib.lib.glt_gemm_pair_mode(-1) == 1
    roofline = {
        "kernel": ("tc_gemm_pair_kernel<6,K,K,EpiSwiGLUFwd> (gate/up GEMM + fused SwiGLU, CTA pairs)" if pair
                   else "tc_gemm_kernel<256,4,K,K,EpiSwiGLUFwd> (gate/up GEMM + fused SwiGLU)"),
        "bound": "tensor", "achieved": achieved, "peak": pk["tf_sus"], "unit": "TFLOP/s",
        "frac": achieved / pk["tf_sus"],
        "peak_note": f"{pk['src']} bf16_tflops_sustained (kernel timed inside a long step)",
        "traffic": GATE_UP_TRAFFIC_BYTES[(pair, bool(store_on))],
        "algorithmic_flops_per_launch": gu_flops, "avg_launch_ms": gu_ms,
        "timing": "CUDA events around every launch on its stream, over a second pass of the "
                  f"same {args.steps} steps ({profiled_ms:.1f} ms per step with the events)",
        "mlp_gemm": {
            "pct_of_peak_algorithmic": 100.0 * mlp_alg / (mlp_ms / 1e3) / 1e12 / pk["tf_sus"],
            "pct_of_burst_peak_algorithmic": 100.0 * mlp_alg / (mlp_ms / 1e3) / 1e12 / pk["tf"],
            "peak_note": "pct_of_peak against the sustained measured bf16 peak; "
                         "pct_of_burst_peak against the burst one",
            "executed_tflops": mlp_exec / (mlp_ms / 1e3) / 1e12,
            "ms_per_step": mlp_ms,
            "definition": "(12*D*F' + 6*D*S) * tokens * layers / time of all MLP GEMM kernels "
                          "(a recompute's time included, its FLOPs not)",
        },
    }
    kernels = {n: {"ms_per_step": kms[i] / args.steps, "launches_per_step": kn[i] / args.steps}
               for i, n in enumerate(G.PROF_NAMES) if kn[i]}

    # e2e: public API with pinned host buffers, stats read back every step
    e2e = None
    if not args.no_e2e:
        h_ids = ids.cpu().pin_memory()
        h_ood = ood.cpu().pin_memory()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.train_step(h_ids, h_ood, step, total_steps + 2 * args.steps, want_stats=True)
            step += 1
        torch.cuda.synchronize()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
        e2e = {"value": tokens_per_step / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": 2 * M * 4, "d2h_bytes_per_step": 32}

    # The same step with the reference's FFN recompute (recompute_ffn) instead
    # of stored pre-activations, timed the same way after the main region.
    extra = {}
    rsteps = args.steps if args.recompute_steps is None else args.recompute_steps
    if store_on and rsteps > 0:
        model.mlp_store(0)
        model.train_step(ids, ood, step, total_steps + 2 * args.steps + rsteps + 1, want_stats=False)
        step += 1
        barrier()
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(rsteps):
            model.train_step(ids, ood, step, total_steps + 2 * args.steps + rsteps + 1, want_stats=False)
            step += 1
        r1.record(stream)
        torch.cuda.synchronize()
        rms = max_over_ranks(r0.elapsed_time(r1) / rsteps)
        extra = {"recompute_ms_per_step": rms, "recompute_tokens_per_s": tokens_per_step / (rms / 1e3),
                 "recompute_steps": rsteps,
                 "recompute_note": "same step with the FFN gate/up recomputed in the backward "
                                   "(recompute_ffn) instead of stored, timed after the main region"}
    if world > 1:
        model.dp_finalize()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, cores = cpu_oracle_sample(wl, args.cpu_tokens)
        cpu = {"value": args.cpu_tokens / (sec * L), "unit": "tokens/s", "cores": cores,
               "kind": "port", "extrapolated": True,
               "sample": f"fp32 CPU oracle: one grafted decoder layer forward+backward on "
                         f"1x{args.cpu_tokens} tokens (median of 2 after 1 warm-up), extrapolated "
                         f"to {L} layers (LM head excluded)"}

    # bf16 weights the step streams (attention, fused MLP, embeddings / LM head)
    Dm, nhm, nkvm, hdm = wl["hidden_dim"], wl["num_heads"], wl["num_kv_heads"], wl["head_dim"]
    w_layer = Dm * (nhm + 2 * nkvm) * hdm + nhm * hdm * Dm + 3 * Dm * (wl["intermediate_dim"] + wl["slice_dim"])
    w_bytes = 2 * (L * w_layer + (1 if wl["tie_embeddings"] else 2) * wl["vocab_size"] * Dm)
    nccl = nccl_summary(nccl_log) if (nccl_log and rank == 0) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform-random token ids, seeded N(0,0.02) random-init weights",
            "config": {"workload": wl["label"], "global_batch": world * B, "seq_len": T,
                       "parallelism": f"dp{world}", "graft": "concat [base | graft], gate+up+down",
                       "mlp_activations": (f"stored: bf16 gate_pre/up of every layer, {store_bytes / 1e9:.1f} GB"
                                           if store_on else "recomputed in the backward (recompute_ffn)"),
                       "l2": f"no flush: the step streams {w_bytes / 1e9:.1f} GB of weights, and its "
                             f"activations, through the 126 MB L2"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "extra": extra,
            "clocks": clk.summary(),
            "gpu_launches": int(launches1.value - launches0.value),
            "kernels": kernels,
        }
        if world > 1:
            line["nccl"] = nccl
            line["dp"] = {"bucket_layers": int(os.environ.get("GLT_DP_BUCKET_LAYERS", "4")),
                          "comm_priority": os.environ.get("GLT_DP_COMM_PRIORITY", "default"),
                          "gemm_schedule": os.environ.get("GLT_GEMM_SCHEDULE", "static")}
        print(json.dumps(line), flush=True)
    model.close()
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
