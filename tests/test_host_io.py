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


# ---------------------------------------------------------------------------
# Training state (fp32 graft + Adam moments + next step): a format of this
# build (the reference keeps only the bf16 deltas), so the checks are exact
# round trips, the header's contents and the refusals.
# ---------------------------------------------------------------------------
def state_arrays(n, seed=3):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(n).astype(np.float32) for _ in range(3)]


def state_save(path, arrs, step=7, session="sess", domain=1, S=4, H=8, D=32, L=2):
    w, m, v = arrs
    return lib.glt_train_state_save(path.encode(), _ptr(w), _ptr(m), _ptr(v), w.size, 1, session.encode(),
                                    domain, S, H, D, L, step)


def state_load(path, n, session="sess", domain=1, S=4, H=8, L=2, fill=0.0):
    outs = [np.full(n, fill, np.float32) for _ in range(3)]
    step = C.c_int64(-1)
    st = lib.glt_train_state_load(path.encode(), _ptr(outs[0]), _ptr(outs[1]), _ptr(outs[2]), n, 1,
                                  session.encode(), domain, 3 * L, S, H, C.byref(step))
    return st, outs, step.value


def test_train_state_roundtrip_is_exact(tmp_path):
    arrs = state_arrays(3 * 2 * 4 * 8)
    arrs[0][5] = np.float32(np.nan)           # bit patterns survive, NaN included
    arrs[1][0] = np.float32(-0.0)
    p = str(tmp_path / "run.state")
    assert state_save(p, arrs, step=123) == 0, _lib.last_error()
    st, outs, step = state_load(p, arrs[0].size)
    assert st == 0 and step == 123, _lib.last_error()
    for a, b in zip(arrs, outs):
        assert a.tobytes() == b.tobytes()


def test_train_state_bytes(tmp_path):
    n = 3 * 2 * 4 * 8
    arrs = state_arrays(n)
    p = str(tmp_path / "run.state")
    assert state_save(p, arrs, step=9, session='a"b') == 0
    blob = open(p, "rb").read()
    assert blob[:4] == b"GLTS" and blob[4] == 1
    hlen = struct.unpack("<Q", blob[5:13])[0]
    assert hlen % 8 == 0
    import json
    hdr = json.loads(blob[13:13 + hlen].rstrip(b"\0"))
    meta = hdr["__metadata__"]
    assert meta == {"format": "glt-train-state", "session_id": 'a"b', "domain_id": "1", "slice_dim": "4",
                    "h_slice_dim": "8", "hidden_dim": "32", "num_layers": "2", "step": "9"}
    data = blob[13 + hlen:]
    assert len(data) == 3 * n * 4
    for k, (name, a) in enumerate(zip(("weights", "adam_m", "adam_v"), arrs)):
        assert hdr[name] == {"dtype": "F32", "shape": [6, 4, 8], "data_offsets": [k * n * 4, (k + 1) * n * 4]}
        assert data[k * n * 4:(k + 1) * n * 4] == a.astype("<f4").tobytes()


@pytest.mark.parametrize("case", ["domain", "session", "shape", "dtype", "truncated", "missing", "grft",
                                  "format"])
def test_train_state_load_rejections_leave_buffers(tmp_path, case):
    n = 3 * 2 * 4 * 8
    arrs = state_arrays(n)
    p = str(tmp_path / "run.state")
    assert state_save(p, arrs) == 0
    kw = {}
    if case == "domain":
        kw["domain"] = 0
    elif case == "session":
        kw["session"] = "other"
    elif case == "shape":
        kw["S"] = 5
    elif case == "dtype":
        blob = open(p, "rb").read().replace(b'"F32"', b'"F16"', 1)
        open(p, "wb").write(blob)
    elif case == "truncated":
        blob = open(p, "rb").read()
        open(p, "wb").write(blob[:-4])
    elif case == "missing":
        p = str(tmp_path / "nope.state")
    elif case == "grft":
        assert save(p, arrs[0]) == 0            # a GRFT checkpoint is not a training state
    elif case == "format":
        blob = open(p, "rb").read().replace(b"glt-train-state", b"glt-train-stat_", 1)
        open(p, "wb").write(blob)
    m = n if case != "shape" else 3 * 2 * 5 * 8
    st, outs, step = state_load(p, m, fill=2.5, **kw)
    assert st in (1, 4), (case, st)
    assert step == -1
    assert all(np.all(o == 2.5) for o in outs)   # untouched on failure


def test_train_state_save_refusals(tmp_path):
    arrs = state_arrays(3 * 2 * 4 * 8)
    assert state_save(str(tmp_path), arrs) == 4
    assert state_save(str(tmp_path / "no" / "dir" / "x.state"), arrs) == 4
    assert state_save(str(tmp_path / "x.state"), arrs, step=-1) == 1
    bad = [a[:-1] for a in arrs]
    assert state_save(str(tmp_path / "x.state"), bad) == 1
