"""Bit-exact CPU restatement of the reference's integer/byte-level pieces.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA library;
only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import it.  The product path never calls it.

Every function cites the reference (Hinedes/GLT) file:line it restates.
Parity is pinned against the reference's own golden vectors in
tests/golden/ (see tests/test_oracle_golden.py).
"""
from __future__ import annotations

import json
import math
import struct

import numpy as np

PROJECTIONS_PER_LAYER = 3          # src/config.hpp:25
GRFT_MAGIC = 0x54465247            # "GRFT" little-endian u32 (src/checkpoint.hpp)
GRFT_VERSION = 4


# ---------------------------------------------------------------------------
# bf16 (src/kernels_elementwise_impl.inc:575-580, src/gemm_impl.inc:69-80)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(x) -> np.ndarray:
    """Bias-trick rounding: bits += ((bits >> 16) & 1) + 0x7FFF; take the top half.

    Equals IEEE round-to-nearest-even for finite values; NaN payloads may wrap
    (the reference has no NaN special case).
    """
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = a.view(np.uint32).astype(np.uint64)
    bits = (bits + ((bits >> 16) & 1) + 0x7FFF) & 0xFFFFFFFF
    return (bits >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    """src/kernels_elementwise_impl.inc:570-573: shift left 16, reinterpret."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---------------------------------------------------------------------------
# Flat graft layout (src/graft_ops_impl.inc:5-7)
# ---------------------------------------------------------------------------
def delta_offset(layer_idx: int, proj_idx: int, slice_dim: int, h_slice_dim: int) -> int:
    """(l*3 + p) * S * H, computed in 64-bit (the reference uses int)."""
    return (layer_idx * PROJECTIONS_PER_LAYER + proj_idx) * slice_dim * h_slice_dim


# ---------------------------------------------------------------------------
# Shadow bake (src/shadow_bake_impl.inc:15-128)
# ---------------------------------------------------------------------------
def shadow_bake_kernel(base_bits: np.ndarray, graft: np.ndarray, i_start: int, h_start: int,
                       mode: int) -> None:
    """In-place bf16 base += f32 delta, reference orientation.

    mode 0 (expand, gate/up):  base[i_start+s, h_start+h] = bf16(base + graft[s,h])
    mode 1 (contract, down):   base[h_start+h, i_start+s] = bf16(base + graft[s,h])
    (src/shadow_bake_impl.inc:15-51).  `base_bits` is a uint16 [rows, cols] array.
    """
    S, H = graft.shape
    if mode == 0:
        view = base_bits[i_start:i_start + S, h_start:h_start + H]
        upd = bf16_bits_to_f32(view) + graft.astype(np.float32)
    else:
        view = base_bits[h_start:h_start + H, i_start:i_start + S]
        upd = bf16_bits_to_f32(view) + graft.astype(np.float32).T
    view[...] = f32_to_bf16_bits(upd.astype(np.float32))


class ShadowBakeState:
    """Mirror of the g_shadow_baked guard (src/shadow_bake.hpp:5)."""

    def __init__(self):
        self.baked = False


def apply_graft_to_shadow(layers: list[dict], graft: np.ndarray | None, cfg, state: ShadowBakeState,
                          domain_id: int) -> None:
    """src/shadow_bake_impl.inc:58-128.

    `layers[l]` holds uint16 arrays 'gate' [F,D], 'up' [F,D], 'down' [D,F];
    `graft` is the flat f32 [3L*S*H] delta buffer (None = empty graft).
    Raises RuntimeError on a second bake (the reference throws).
    """
    if state.baked:
        raise RuntimeError("apply_graft_to_shadow called twice on the same model instance")
    state.baked = True
    if graft is None:
        return
    S, H = cfg.slice_dim, cfg.h_slice_dim
    i_start, h_start = domain_id * S, domain_id * H
    for l in range(cfg.num_layers):
        if not (cfg.graft_layer_start <= l <= cfg.graft_layer_end):
            continue
        for p, name, mode, flag in ((0, "gate", 0, cfg.graft_proj_gate),
                                    (1, "up", 0, cfg.graft_proj_up),
                                    (2, "down", 1, cfg.graft_proj_down)):
            if not flag:
                continue
            off = delta_offset(l, p, S, H)
            g = graft[off:off + S * H].reshape(S, H)
            shadow_bake_kernel(layers[l][name], g, i_start, h_start, mode)


# ---------------------------------------------------------------------------
# GRFT checkpoint (src/checkpoint_impl.inc:8-89, 170-285)
# ---------------------------------------------------------------------------
def build_safetensors_header(session_id: str, domain_id: int, slice_dim: int, h_slice_dim: int,
                             hidden_dim: int, num_layers: int) -> str:
    """src/checkpoint_impl.inc:8-30 (key order and formatting kept byte-for-byte)."""
    total_proj = num_layers * PROJECTIONS_PER_LAYER
    nbytes = total_proj * slice_dim * h_slice_dim * 2
    return (
        "{"
        "\"__metadata__\":{"
        f"\"session_id\":\"{session_id}\","
        f"\"domain_id\":\"{domain_id}\","
        f"\"slice_dim\":\"{slice_dim}\","
        f"\"h_slice_dim\":\"{h_slice_dim}\","
        f"\"hidden_dim\":\"{hidden_dim}\","
        f"\"num_layers\":\"{num_layers}\""
        "},"
        "\"delta_weights\":{"
        "\"dtype\":\"BF16\","
        f"\"shape\":[{total_proj},{slice_dim},{h_slice_dim}],"
        f"\"data_offsets\":[0,{nbytes}]"
        "}"
        "}"
    )


def grft_bytes(weights_f32: np.ndarray, session_id: str, domain_id: int, slice_dim: int,
               h_slice_dim: int, hidden_dim: int, num_layers: int) -> bytes:
    """Byte image of save_safetensors (src/checkpoint_impl.inc:32-89):
    u32 'GRFT' | u8 version 4 | u64 header_size (JSON padded with NUL to 8) | JSON | BF16 data.
    """
    header = build_safetensors_header(session_id, domain_id, slice_dim, h_slice_dim, hidden_dim,
                                      num_layers).encode()
    pad = (8 - len(header) % 8) % 8
    body = f32_to_bf16_bits(np.asarray(weights_f32, dtype=np.float32).ravel()).tobytes()
    return (struct.pack("<IBQ", GRFT_MAGIC, GRFT_VERSION, len(header) + pad) + header +
            b"\x00" * pad + body)


class CheckpointError(Exception):
    pass


def parse_grft(buf: bytes, expected_domain_id: int, session_id: str, total_projections: int,
               slice_dim: int, h_slice_dim: int) -> np.ndarray:
    """load_safetensors_checkpoint (src/checkpoint_impl.inc:170-285) -> f32 weights.

    Accepts the GRFT prefix or a legacy plain safetensors file; validates dtype,
    shape, session_id and domain_id exactly as the reference does.
    """
    off = 0
    if len(buf) >= 5 and struct.unpack_from("<I", buf, 0)[0] == GRFT_MAGIC:
        off = 5
    st = buf[off:]
    if len(st) < 8:
        raise CheckpointError("safetensors parse failed: too small")
    (hlen,) = struct.unpack_from("<Q", st, 0)
    if 8 + hlen > len(st):
        raise CheckpointError("safetensors parse failed: header past end of file")
    try:
        hdr = json.loads(st[8:8 + hlen].rstrip(b"\x00 ").decode())
    except Exception as e:  # noqa: BLE001
        raise CheckpointError(f"safetensors parse failed: {e}") from e
    if "delta_weights" not in hdr:
        raise CheckpointError("'delta_weights' not found")
    t = hdr["delta_weights"]
    if t.get("dtype") != "BF16":
        raise CheckpointError("delta_weights dtype is not BF16")
    shape = t.get("shape", [])
    if list(shape) != [total_projections, slice_dim, h_slice_dim]:
        raise CheckpointError(f"delta_weights shape mismatch: {shape}")
    meta = hdr.get("__metadata__", {})
    file_session = meta.get("session_id", "")
    if session_id and file_session and session_id != file_session:
        raise CheckpointError("session_id mismatch")
    if "domain_id" in meta and int(meta["domain_id"]) != expected_domain_id:
        raise CheckpointError("checkpoint domain_id mismatch")
    b0, b1 = t["data_offsets"]
    data = st[8 + hlen + b0: 8 + hlen + b1]
    n = total_projections * slice_dim * h_slice_dim
    if len(data) < 2 * n:
        raise CheckpointError("truncated tensor data")
    return bf16_bits_to_f32(np.frombuffer(data[:2 * n], dtype=np.uint16))


# ---------------------------------------------------------------------------
# .bin token files (src/data_impl.inc:9-58)
# ---------------------------------------------------------------------------
class BinError(Exception):
    pass


def parse_bin(buf: bytes) -> tuple[int, int, np.ndarray]:
    """[i32 num_sequences][i32 seq_len][i32 tokens...] with the reference's checks."""
    if len(buf) < 8:
        raise BinError("failed reading header")
    n, t = struct.unpack_from("<ii", buf, 0)
    if n <= 0 or t <= 0:
        raise BinError("invalid header")
    total = n * t
    if total > (1 << 30):
        raise BinError("token count exceeds safety limit")
    if len(buf) - 8 < total * 4:
        raise BinError("truncated token data")
    toks = np.frombuffer(buf[8:8 + total * 4], dtype="<i4").astype(np.int32)
    return n, t, toks


# ---------------------------------------------------------------------------
# Batch walk (grafting.hip:924-988)
# ---------------------------------------------------------------------------
MASK64 = (1 << 64) - 1


def mix_seed(x: int) -> int:
    """splitmix64 finaliser, grafting.hip:928-933."""
    x = (x + 0x9E3779B97F4A7C15) & MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return x ^ (x >> 31)


def batch_walk_start(seed: int, n_domain: int, n_ood: int) -> tuple[int, int]:
    """grafting.hip:935-937: initial corpus positions from the seed."""
    s = seed & MASK64
    return mix_seed(s) % n_domain, mix_seed(s ^ 0x9E3779B97F4A7C15) % n_ood


def batch_step(domain_tokens: np.ndarray, n_domain: int, ood_tokens: np.ndarray, n_ood: int,
               seq_len: int, batch_size: int, domain_pos: int, ood_pos: int):
    """One step of grafting.hip:965-983: first half domain rows, second half OOD rows.

    Returns (ids [B*T] int32, ood_mask [B*T] int32, new_domain_pos, new_ood_pos).
    """
    half = batch_size // 2
    ids = np.empty(batch_size * seq_len, dtype=np.int32)
    mask = np.empty(batch_size * seq_len, dtype=np.int32)
    for i in range(half):
        ds = (domain_pos + i) % n_domain
        ids[i * seq_len:(i + 1) * seq_len] = domain_tokens[ds * seq_len:(ds + 1) * seq_len]
        mask[i * seq_len:(i + 1) * seq_len] = 0
    domain_pos = (domain_pos + half) % n_domain
    for i in range(half):
        os_ = (ood_pos + i) % n_ood
        ids[(half + i) * seq_len:(half + i + 1) * seq_len] = ood_tokens[os_ * seq_len:(os_ + 1) * seq_len]
        mask[(half + i) * seq_len:(half + i + 1) * seq_len] = 1
    ood_pos = (ood_pos + half) % n_ood
    return ids, mask, domain_pos, ood_pos


# ---------------------------------------------------------------------------
# LR schedule (src/config.hpp:122-129), float32 arithmetic as in the reference
# ---------------------------------------------------------------------------
def get_lr(step: int, total_steps: int, lr_peak: float, warmup: int) -> float:
    f32 = np.float32
    if step < warmup:
        return float(f32(f32(lr_peak) * f32(step + 1)) / f32(warmup))
    denom = f32(total_steps - warmup)
    progress = f32(f32(step - warmup) / max(denom, f32(1.0)))
    arg = f32(math.pi * float(progress))          # cosf(M_PI * progress): float argument
    c = f32(math.cos(float(arg)))
    return float(f32(f32(f32(lr_peak) * f32(f32(1.0) + c)) * f32(0.5)))


# ---------------------------------------------------------------------------
# FNV-1a 64 over little-endian fp32 logits (grafting.hip:504, 535-547)
# ---------------------------------------------------------------------------
def fnv1a64_f32(values: np.ndarray, h: int = 1469598103934665603) -> int:
    data = np.ascontiguousarray(values, dtype="<f4").reshape(-1).view(np.uint8)
    for byte in data.tolist():
        h ^= byte
        h = (h * 1099511628211) & MASK64
    return h
