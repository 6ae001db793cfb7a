"""Helpers of the graft_train command-line tests: writers for the two input
formats the reference reads (Hugging Face safetensors shards and the .bin
token files of src/data_impl.inc:9-58) and a runner for the binary."""
from __future__ import annotations

import json
import os
import struct
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "glt_b200", "graft_train")


def write_safetensors(path: str, tensors: dict[str, np.ndarray], dtypes: dict[str, str] | None = None):
    """tensors: name -> fp32 array; dtypes: name -> "BF16" (default), "F32" or "F16"."""
    from oracle.bitexact import f32_to_bf16_bits
    dtypes = dtypes or {}
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, arr in tensors.items():
        dt = dtypes.get(name, "BF16")
        a = np.ascontiguousarray(arr, dtype=np.float32)
        if dt == "BF16":
            raw = f32_to_bf16_bits(a).astype("<u2").tobytes()
        elif dt == "F16":
            raw = a.astype("<f2").tobytes()
        else:
            raw = a.astype("<f4").tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def hf_tensors(w: dict, tied: bool = True) -> dict[str, np.ndarray]:
    """Oracle weight dict (tests.parity.make_decoder_weights) -> HF names."""
    out = {"model.embed_tokens.weight": w["embed"].numpy(), "model.norm.weight": w["final_norm"].numpy()}
    for l, lw in enumerate(w["layers"]):
        p = f"model.layers.{l}."
        out[p + "input_layernorm.weight"] = lw["in_norm"].numpy()
        out[p + "self_attn.q_proj.weight"] = lw["wq"].numpy()
        out[p + "self_attn.k_proj.weight"] = lw["wk"].numpy()
        out[p + "self_attn.v_proj.weight"] = lw["wv"].numpy()
        out[p + "self_attn.o_proj.weight"] = lw["wo"].numpy()
        out[p + "post_attention_layernorm.weight"] = lw["post_norm"].numpy()
        out[p + "mlp.gate_proj.weight"] = lw["wg"].numpy()
        out[p + "mlp.up_proj.weight"] = lw["wu"].numpy()
        out[p + "mlp.down_proj.weight"] = lw["wd"].numpy()
    if not tied:
        out["lm_head.weight"] = w["lm_head"].numpy()
    return out


def write_bin(path: str, tokens: np.ndarray):
    """[i32 num_sequences][i32 seq_len][i32 tokens...]"""
    t = np.ascontiguousarray(tokens, dtype="<i4")
    with open(path, "wb") as f:
        f.write(struct.pack("<ii", t.shape[0], t.shape[1]))
        f.write(t.tobytes())


def run_cli(*args, timeout: int = 600) -> subprocess.CompletedProcess:
    return subprocess.run([CLI, *map(str, args)], capture_output=True, text=True, timeout=timeout)


def key_values(stdout: str) -> dict[str, str]:
    kv = {}
    for line in stdout.splitlines():
        if "=" in line and not line.startswith((" ", "[")):
            k, v = line.split("=", 1)
            kv[k.strip()] = v.strip()
    return kv
