"""GRFT checkpoint, .bin loader and batch walk through the C ABI, byte-exact
against the oracle (CPU only: host buffers)."""
import ctypes as C
import os
import struct

import numpy as np
import pytest

from glt_b200 import _lib
from oracle import bitexact as bx

lib = _lib.lib


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def save(path, w, session="sess", domain=1, S=4, H=8, D=32, L=2):
    return lib.glt_checkpoint_save(path.encode(), _ptr(w), w.size, 1, session.encode(), domain, S, H, D, L)


def load(path, n, domain=1, session="sess", S=4, H=8, L=2):
    out = np.zeros(n, np.float32)
    fd = C.c_int(-7)
    st = lib.glt_checkpoint_load(path.encode(), _ptr(out), n, 1, domain, session.encode(), 3 * L, S, H,
                                 C.byref(fd))
    return st, out, fd.value


def test_checkpoint_bytes_match_oracle(tmp_path):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(3 * 2 * 4 * 8) * 0.1).astype(np.float32)
    p = str(tmp_path / "g.graft")
    assert save(p, w) == 0, _lib.last_error()
    assert open(p, "rb").read() == bx.grft_bytes(w, "sess", 1, 4, 8, 32, 2)


def test_checkpoint_roundtrip_is_bf16_rounding(tmp_path):
    rng = np.random.default_rng(1)
    w = rng.standard_normal(3 * 2 * 4 * 8).astype(np.float32)
    p = str(tmp_path / "g.graft")
    assert save(p, w) == 0
    st, back, fd = load(p, w.size)
    assert st == 0 and fd == 1
    np.testing.assert_array_equal(back, bx.round_bf16(w))


@pytest.mark.parametrize("case", ["domain", "session", "shape", "dtype", "truncated", "missing"])
def test_checkpoint_load_rejections(tmp_path, case):
    w = np.zeros(3 * 2 * 4 * 8, np.float32)
    p = str(tmp_path / "g.graft")
    assert save(p, w) == 0
    kw = {}
    if case == "domain":
        kw["domain"] = 0
    elif case == "session":
        kw["session"] = "other"
    elif case == "shape":
        kw["S"] = 5
    elif case == "dtype":
        blob = open(p, "rb").read().replace(b'"BF16"', b'"F32\x20"')
        open(p, "wb").write(blob)
    elif case == "truncated":
        blob = open(p, "rb").read()
        open(p, "wb").write(blob[:-3])
    elif case == "missing":
        p = str(tmp_path / "nope.graft")
    n = w.size if case != "shape" else 3 * 2 * 5 * 8
    st, _, _ = load(p, n, **kw)
    assert st in (1, 4), (case, st)


def test_checkpoint_legacy_and_missing_domain(tmp_path):
    w = np.arange(3 * 2 * 4 * 8, dtype=np.float32) / 64.0
    legacy = bx.grft_bytes(w, "", 0, 4, 8, 32, 2)[5:]
    p = str(tmp_path / "legacy.safetensors")
    open(p, "wb").write(legacy)
    st, back, fd = load(p, w.size, domain=0, session="")
    assert st == 0 and fd == 0
    np.testing.assert_array_equal(back, bx.round_bf16(w))


def test_checkpoint_save_refuses_directory_and_missing_parent(tmp_path):
    w = np.zeros(3 * 2 * 4 * 8, np.float32)
    assert save(str(tmp_path), w) == 4
    assert save(str(tmp_path / "no" / "such" / "dir.graft"), w) == 4


def write_bin(path, nseq, T, toks=None):
    toks = np.arange(nseq * T, dtype=np.int32) if toks is None else toks
    open(path, "wb").write(struct.pack("<ii", nseq, T) + toks.astype("<i4").tobytes())
    return toks


def test_load_bin_roundtrip(tmp_path):
    p = str(tmp_path / "d.bin")
    toks = write_bin(p, 3, 5)
    n, t = C.c_int32(), C.c_int32()
    assert lib.glt_load_bin(p.encode(), C.byref(n), C.byref(t), None, 0) == 0
    assert (n.value, t.value) == (3, 5)
    out = np.zeros(15, np.int32)
    assert lib.glt_load_bin(p.encode(), C.byref(n), C.byref(t), _ptr(out), out.size) == 0
    np.testing.assert_array_equal(out, toks)
    nn, tt, ref = bx.parse_bin(open(p, "rb").read())
    np.testing.assert_array_equal(out, ref)


@pytest.mark.parametrize("hdr,extra", [((0, 5), 64), ((-2, 5), 64), ((3, 0), 64), ((3, 5), 59)])
def test_load_bin_rejects(tmp_path, hdr, extra):
    p = str(tmp_path / "bad.bin")
    open(p, "wb").write(struct.pack("<ii", *hdr) + b"\x01" * extra)
    n, t = C.c_int32(), C.c_int32()
    assert lib.glt_load_bin(p.encode(), C.byref(n), C.byref(t), None, 0) == 4


def test_batch_walk_matches_oracle():
    T, nd, no, B = 6, 5, 3, 4
    rng = np.random.default_rng(3)
    dom = rng.integers(0, 1000, nd * T).astype(np.int32)
    ood = rng.integers(0, 1000, no * T).astype(np.int32)
    dp, op = C.c_int(), C.c_int()
    assert lib.glt_batch_walk_start(42, nd, no, C.byref(dp), C.byref(op)) == 0
    rdp, rop = bx.batch_walk_start(42, nd, no)
    assert (dp.value, op.value) == (rdp, rop)
    ids = np.zeros(B * T, np.int32)
    mask = np.zeros(B * T, np.int32)
    for _ in range(4):
        assert lib.glt_batch_step(_ptr(dom), nd, _ptr(ood), no, T, B, C.byref(dp), C.byref(op),
                                  _ptr(ids), _ptr(mask)) == 0
        rids, rmask, rdp, rop = bx.batch_step(dom, nd, ood, no, T, B, rdp, rop)
        np.testing.assert_array_equal(ids, rids)
        np.testing.assert_array_equal(mask, rmask)
        assert (dp.value, op.value) == (rdp, rop)


def test_batch_step_rejects_odd_batch():
    a = np.zeros(8, np.int32)
    dp, op = C.c_int(0), C.c_int(0)
    assert lib.glt_batch_step(_ptr(a), 1, _ptr(a), 1, 4, 3, C.byref(dp), C.byref(op), _ptr(a), _ptr(a)) == 1
