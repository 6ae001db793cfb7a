"""Causal GQA attention microbench (default: the attention of the Llama-3-8B decoder layer).

    python -m glt_b200.attn_bench [--batch 16] [--seq 2048] [--heads 32] [--kv-heads 8]
                                  [--head-dim 128] [--impl tc|mma] [--steps 10] [--warmup 3]

Times glt_attention_fwd and glt_attention_bwd (the C ABI the decoder calls)
with CUDA events on the launching stream and prints one JSON line with the
per-call time and the algorithmic TFLOP/s of each direction.  Algorithmic
FLOPs of causal attention (the reference runs SDPA with is_causal,
layer_forward_impl.inc:41-49): forward 4*B*nh*hd*T*(T+1)/2 (QK^T and PV over
the visible half), backward 2.5x that (S and dP recomputed, dV, dK, dQ).
The inputs (q/k/v 0.4 GB at the default shape) exceed the 126 MB L2.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

import torch

from . import _lib


def run(B: int, T: int, nh: int, nkv: int, hd: int, impl: int, steps: int, warmup: int) -> dict:
    lib = _lib.lib
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(7)
    QKV = (nh + 2 * nkv) * hd
    qkv = torch.randn(B * T, QKV, device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, nh, T, device=dev)
    dout = torch.randn(B * T, nh * hd, device=dev, generator=g).to(torch.bfloat16)
    dqkv = torch.zeros_like(qkv)
    dq_acc = torch.empty(B * T * (nh + 2 * nkv) * hd, device=dev)   # dQ (+ dK/dV at hd 64, tcgen05)
    dsum = torch.empty(B * nh * T, device=dev)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)

    def vp(t):
        return C.c_void_p(t.data_ptr())

    def fwd():
        _lib.check(lib.glt_attention_fwd(vp(qkv), QKV, vp(o), nh * hd, vp(lse), B, T, nh, nkv, hd,
                                         impl, sp))

    def bwd():
        _lib.check(lib.glt_attention_bwd(vp(qkv), QKV, vp(o), vp(dout), nh * hd, vp(lse), vp(dqkv),
                                         vp(dq_acc), vp(dsum), B, T, nh, nkv, hd, impl, sp))

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    fwd()
    ms_f = timed(fwd)
    ms_b = timed(bwd)
    dev_err = C.c_uint()
    _lib.check(lib.glt_device_error(C.byref(dev_err)))
    flops_f = 4.0 * B * nh * hd * T * (T + 1) / 2
    flops_b = 2.5 * flops_f
    return {"batch": B, "seq": T, "heads": nh, "kv_heads": nkv, "head_dim": hd,
            "impl": "tcgen05" if impl == 0 else "mma.sync",
            "fwd_ms": ms_f, "fwd_tflops": flops_f / (ms_f / 1e3) / 1e12,
            "bwd_ms": ms_b, "bwd_tflops": flops_b / (ms_b / 1e3) / 1e12,
            "bwd_includes": "dsum prep + fp32 dQ (hd 64: and dK/dV) reduce + bf16 convert",
            "device_error": dev_err.value}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--impl", choices=["tc", "mma"], default="tc")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    r = run(a.batch, a.seq, a.heads, a.kv_heads, a.head_dim, 0 if a.impl == "tc" else 1, a.steps,
            a.warmup)
    print(json.dumps(r), flush=True)
    return 0 if r["device_error"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
