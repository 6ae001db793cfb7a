"""The row-parallel evaluation of the reference's logits fingerprint.

The reference hashes the fp32 bytes of all eval logits with sequential
FNV-1a 64 (grafting.hip:504, 535-547).  The GPU evaluates it row-parallel
through an exact identity of FNV-1a: XOR with a byte changes only the low
byte of the state, and multiplying by the prime keeps the low byte a function
of the low byte, so for a byte string of length n

    F(h) = F(h mod 256) + (h - h mod 256) * P^n   (mod 2^64).

Each row therefore needs only the 256 values F(s), s = 0..255 (one GPU thread
each), and a sequential fold over rows.  These tests check that algebra
against the oracle's sequential hash, on bf16-valued logits (whose two low
fp32 bytes are zero, the case the kernel specialises) and on general floats.
"""
import numpy as np

from oracle.bitexact import MASK64, fnv1a64_f32, round_bf16

P = 1099511628211
BASIS = 1469598103934665603


def row_table(row_bytes: bytes) -> list[int]:
    out = []
    for s in range(256):
        h = s
        for b in row_bytes:
            h = ((h ^ b) * P) & MASK64
        out.append(h)
    return out


def split_hash(values: np.ndarray, h: int = BASIS) -> int:
    rows = np.ascontiguousarray(values, dtype="<f4")
    pn = pow(P, 4 * rows.shape[1], 1 << 64)
    for r in rows:
        t = row_table(r.view(np.uint8).tobytes())
        s = h & 255
        h = (t[s] + (h - s) * pn) & MASK64
    return h


def test_split_hash_equals_sequential_fnv_on_bf16_logits():
    rng = np.random.default_rng(0)
    x = round_bf16(rng.standard_normal((5, 7)).astype(np.float32) * 4)
    assert split_hash(x) == fnv1a64_f32(x)


def test_split_hash_equals_sequential_fnv_on_general_floats():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 5)).astype(np.float32)
    assert split_hash(x) == fnv1a64_f32(x)
    # chaining over batches: the fold continues from the previous state
    y = rng.standard_normal((2, 5)).astype(np.float32)
    assert split_hash(y, split_hash(x)) == fnv1a64_f32(np.concatenate([x, y]))


def test_zero_bytes_are_a_plain_multiply():
    # bf16 logits stored as fp32 have two zero low bytes: (h ^ 0) * P = h * P
    h = 0x0123456789ABCDEF
    assert ((h ^ 0) * P * P) & MASK64 == (h * ((P * P) & MASK64)) & MASK64
