"""Builds the in-tree shared library glt_b200/libglt_b200.so for sm_100a.

Every CUDA/C++ source under glt_b200/csrc is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared
library with the CUDA runtime linked statically, so the library carries no
link-time dependency on libcuda (the driver entry points it needs are
resolved at run time) and loads on GPU-less hosts, where its host-only entry
points (checkpoint format, data loader, config checks) remain callable.

Usage:  python -m glt_b200.build [--force] [-j N] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libglt_b200.so")
CLI_SRC = os.path.join(HERE, "cli", "graft_train.cpp")
CLI = os.path.join(HERE, "graft_train")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(
        os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp"))
    )


def _headers_digest() -> str:
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cuh", ".h", ".hpp")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    return h.hexdigest()


def _obj_path(src: str, digest: str, extra: list[str]) -> str:
    h = hashlib.sha256()
    with open(src, "rb") as fh:
        h.update(fh.read())
    h.update(digest.encode())
    h.update(" ".join(NVCC_FLAGS + ARCH + extra).encode())
    base = os.path.splitext(os.path.basename(src))[0]
    return os.path.join(BUILD, f"{base}-{h.hexdigest()[:16]}.o")


def _compile(src: str, obj: str, extra: list[str]) -> tuple[str, str]:
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + extra + ["-x", "cu", "-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{p.stdout}\n{p.stderr}")
    return src, (p.stdout + p.stderr)


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    digest = _headers_digest()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = sources()
    objs = [_obj_path(s, digest, extra) for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or not os.path.exists(o)]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for src, log in ex.map(lambda so: _compile(so[0], so[1], extra), todo):
                if log.strip():
                    logs.append(f"== {os.path.basename(src)}\n{log}")
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if force or todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest_obj:
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lpthread"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
        os.replace(tmp, LIB)
    # drop stale objects
    keep = set(objs)
    for f in os.listdir(BUILD):
        fp = os.path.join(BUILD, f)
        if fp not in keep and f.endswith(".o"):
            os.remove(fp)
    if logs:
        sys.stderr.write("\n".join(logs) + "\n")
    build_cli(force)
    return LIB


def build_cli(force: bool = False) -> str:
    """The graft_train command line: plain C++ over the C ABI, linked against
    the in-tree library (found next to the binary at run time)."""
    hdr = os.path.join(ROOT, "include", "glt_graft.h")
    newest = max(os.path.getmtime(p) for p in (CLI_SRC, hdr, LIB))
    if not force and os.path.exists(CLI) and os.path.getmtime(CLI) >= newest:
        return CLI
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-I" + os.path.join(ROOT, "include"), CLI_SRC,
           "-o", CLI + ".tmp", "-L" + HERE, "-lglt_b200", "-Wl,-rpath,$ORIGIN"]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"graft_train build failed:\n{p.stdout}\n{p.stderr}")
    os.replace(CLI + ".tmp", CLI)
    return CLI


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose_ptxas=a.verbose_ptxas))


if __name__ == "__main__":
    main()
