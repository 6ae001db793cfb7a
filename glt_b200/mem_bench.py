"""Bandwidth-bound kernels of the grafted decoder step at the config-3 shape.

    python -m glt_b200.mem_bench [--tokens 32768] [--layers 32] [--steps 5] [--warmup 3]

Times each kernel through the C ABI with CUDA events on the launching stream
(warm-up first; every buffer is larger than the 126 MB L2 except where noted)
and prints one JSON line per kernel with its algorithmic bytes, GB/s and the
fraction of the measured HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs).

Algorithmic bytes (bf16 = 2 B, fp32 = 4 B), per unit:
  rmsnorm_fwd   per token: x 2D + y 2D + var 4             (kernels_rmsnorm, K1)
  rmsnorm_bwd   per token: dy 4D + x 2D + resid 4D + dx 4D   (K2, residual fused)
  rope          per token: q and k read + written, 2 B x 2 x (nh + nkv) hd
  swiglu_fwd    per element of [M, F']: gate 2 + up 2 + h 2
  swiglu_bwd    per element: gp 2 + up 2 + grad_h 4 + grad_gp 4 + grad_up 4
  adamw         per graft parameter: w, g, m, v read (16) + w, m, v written (12)
                + bf16 image (2) = 30
  shadow_bake   per graft element: graft 4 + base read 2 + base written 2 = 8,
                over all 3L projections of the model
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

import torch

from . import _lib
from . import graft as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def hbm_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


def vp(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def timed(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", default="")
    a = ap.parse_args(argv)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    lib = _lib.lib
    M, D, F, S, L = a.tokens, 4096, 14336, 1024, a.layers
    Fp = F + S
    nh, nkv, hd, T = 32, 8, 128, 2048
    peak, src = hbm_peak()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(0)
    only = set(a.only.split(",")) if a.only else None
    out = []

    def report(name, ms, nbytes, unit_note):
        gbs = nbytes / (ms / 1e3) / 1e9
        line = {"kernel": name, "ms": round(ms, 4), "bytes": int(nbytes), "gbs": round(gbs, 1),
                "frac_of_hbm": round(gbs / peak, 3), "peak_gbs": peak, "peak_src": src,
                "workload": unit_note}
        out.append(line)
        print(json.dumps(line), flush=True)

    def want(n):
        return only is None or n in only

    if want("rmsnorm_fwd") or want("rmsnorm_bwd"):
        x = torch.randn(M, D, device="cuda", generator=g).to(torch.bfloat16)
        w = torch.ones(D, device="cuda", dtype=torch.bfloat16)
        y = torch.empty_like(x)
        var = torch.empty(M, device="cuda")
        eps = 1e-6
        if want("rmsnorm_fwd"):
            ms = timed(lambda: _lib.check(lib.glt_rmsnorm_fwd(vp(x), vp(w), vp(y), vp(var), M, D, eps, st)),
                       a.steps, a.warmup)
            report("rmsnorm_fwd", ms, M * (4 * D + 4) + 2 * D, f"{M} tokens x D {D}")
        if want("rmsnorm_bwd"):
            _lib.check(lib.glt_rmsnorm_fwd(vp(x), vp(w), vp(y), vp(var), M, D, eps, st))
            dy = torch.randn(M, D, device="cuda", generator=g)
            resid = torch.randn(M, D, device="cuda", generator=g)
            dx = torch.empty(M, D, device="cuda")
            ms = timed(lambda: _lib.check(lib.glt_rmsnorm_bwd(vp(dy), vp(x), vp(w), vp(var), vp(resid),
                                                              vp(dx), M, D, eps, st)), a.steps, a.warmup)
            report("rmsnorm_bwd", ms, M * 14 * D + 2 * D + 4 * M, f"{M} tokens x D {D}, residual fused")
            del dy, resid, dx
        del x, y, var

    if want("rope"):
        QKV = (nh + 2 * nkv) * hd
        qkv = torch.randn(M, QKV, device="cuda", generator=g).to(torch.bfloat16)
        B = M // T
        ms = timed(lambda: _lib.check(lib.glt_rope(vp(qkv), QKV, B, T, nh, nkv, hd, 5e5, 0, st)),
                   a.steps, a.warmup)
        report("rope", ms, M * 4 * (nh + nkv) * hd, f"{B}x{T} tokens, {nh}q/{nkv}kv hd {hd}")
        del qkv

    if want("swiglu_fwd"):
        gu = torch.randn(M, 2 * Fp, device="cuda", generator=g).to(torch.bfloat16)
        h = torch.empty(M, Fp, device="cuda", dtype=torch.bfloat16)
        up = gu[:, Fp:]
        ms = timed(lambda: _lib.check(lib.glt_swiglu_fwd(vp(gu), vp(up), vp(h), M, Fp, 2 * Fp, 2 * Fp,
                                                         Fp, st)), a.steps, a.warmup)
        report("swiglu_fwd", ms, M * Fp * 6, f"[{M}, {Fp}] gate/up strided in one [M, 2F'] buffer")
        del gu, h

    if want("swiglu_bwd"):
        n = M * Fp
        gp = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
        up = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
        gi = torch.randn(n, device="cuda", generator=g)
        dg = torch.empty(n, device="cuda")
        du = torch.empty(n, device="cuda")
        ms = timed(lambda: _lib.check(lib.glt_swiglu_bwd(vp(dg), vp(du), vp(gi), vp(up), vp(gp), n, st)),
                   a.steps, a.warmup)
        report("swiglu_bwd", ms, n * 16, f"{n} elements ([{M}, {Fp}])")
        del gp, up, gi, dg, du

    if want("adamw"):
        cfg = G.GraftConfig(hidden_dim=D, intermediate_dim=F, slice_dim=S, num_layers=L, num_heads=nh,
                            num_kv_heads=nkv, vocab_size=0, layout=G.LAYOUT_CONCAT, graft_layer_start=0,
                            graft_layer_end=L - 1, graft_proj_gate=1, graft_proj_up=1, graft_proj_down=1,
                            allow_expansion_trap=1).to_c()
        n = 3 * L * S * D
        w = torch.randn(n, device="cuda", generator=g) * 0.02
        gr = torch.randn(n, device="cuda", generator=g) * 1e-3
        m = torch.zeros(n, device="cuda")
        v = torch.zeros(n, device="cuda")
        img = torch.empty(n, device="cuda", dtype=torch.int16)
        step = [0]

        def run():
            _lib.check(lib.glt_adamw_all(vp(w), vp(img), vp(gr), vp(m), vp(v), None, C.byref(cfg),
                                         step[0], 1e-4, st))
            step[0] += 1
        ms = timed(run, a.steps, a.warmup)
        report("adamw", ms, n * 30, f"{n} graft parameters (3 x {L} x {S} x {D})")
        del w, gr, m, v, img

    if want("shadow_bake"):
        # the touched part of each base matrix: gate/up rows [S, D] (expand
        # mode, row stride D) and the down block [D, S] (contract mode, row stride S)
        base = torch.randn(3 * L * S * D, device="cuda", generator=g).to(torch.bfloat16)
        graft = torch.randn(3 * L * S * D, device="cuda", generator=g) * 0.02

        def run():
            for l in range(L):
                for p in range(3):
                    off = (3 * l + p) * S * D
                    b = C.c_void_p(base.data_ptr() + 2 * off)
                    src = C.c_void_p(graft.data_ptr() + 4 * off)
                    if p < 2:
                        _lib.check(lib.glt_shadow_bake(b, D, src, S, D, 0, 0, 0, st))
                    else:
                        _lib.check(lib.glt_shadow_bake(b, S, src, S, D, 0, 0, 1, st))
        ms = timed(run, a.steps, a.warmup)
        report("shadow_bake", ms, 3 * L * S * D * 8, f"3 x {L} projections of {S} x {D}")
        del base, graft

    dev_err = C.c_uint()
    _lib.check(lib.glt_device_error(C.byref(dev_err)))
    return 0 if dev_err.value == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
