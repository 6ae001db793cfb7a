"""graft_train flag handling without a GPU: the reference's refusals
(grafting.hip:364-444, 446-470, 590-606, 715-735) happen before any device
work, and the host-side safetensors reader of the base-model loader."""
import os

import numpy as np
import pytest

from glt_b200 import _lib
from tests.cli_util import CLI, run_cli, write_safetensors

pytestmark = pytest.mark.skipif(not os.path.exists(CLI), reason="graft_train not built")

TRAIN = ["--safetensors", "m.safetensors", "--domain-data", "d.bin", "--ood-data", "o.bin",
         "--output", "ck.graft"]


def test_help():
    r = run_cli("--help")
    assert r.returncode == 0 and "--safetensors" in r.stdout and "--graft-layout" in r.stdout


@pytest.mark.parametrize("args,msg", [
    (["--graft-proj-gate", "1", "--graft-proj-up", "1"], "Expansion Quadratic Trap"),
    (["--graft-gemm-backend", "cublas"], "invalid --graft-gemm-backend"),
    (["--graft-layout", "sideways"], "invalid --graft-layout"),
    (["--max-domains", "0"], "--max-domains must be positive"),
    (["--num-heads", "0"], "--num-heads must be positive"),
    (["--domain-id", "4"], "out of range"),
    (["--slice-dim", "2750", "--intermediate-dim", "11000"], "multiple of 4"),
    (["--graft-proj-down", "0"], "no graft projection enabled"),
    (["--graft-proj-down", "2"], "must be 0 or 1"),
    (["--num-layers", "3", "--no-rope-layers", "1,0"], "expects 3 values"),
])
def test_shared_validation(args, msg):
    r = run_cli(*TRAIN, *args)
    assert r.returncode != 0 and msg in r.stderr, r.stderr


def test_training_requires_inputs_and_even_batch(tmp_path):
    r = run_cli("--safetensors", "m.safetensors")
    assert r.returncode != 0 and "are required" in r.stderr
    r = run_cli(*TRAIN[:-1], str(tmp_path))
    assert r.returncode != 0 and "is a directory" in r.stderr
    r = run_cli(*TRAIN[:-1], str(tmp_path / "missing" / "ck.graft"))
    assert r.returncode != 0 and "does not exist" in r.stderr
    r = run_cli(*TRAIN[:-1], str(tmp_path / "ck.graft"), "--batch-size", "3")
    assert r.returncode != 0 and "must be even" in r.stderr


@pytest.mark.parametrize("mode", ["--eval-only", "--shadow-eval"])
def test_eval_modes_refuse_training_flags(mode):
    r = run_cli(mode, "--safetensors", "m", "--eval-data", "e.bin", "--output", "x.graft")
    assert r.returncode != 0 and "does not save a checkpoint" in r.stderr
    r = run_cli(mode, "--safetensors", "m", "--eval-data", "e.bin", "--domain-data", "d.bin")
    assert r.returncode != 0 and "incompatible with --domain-data" in r.stderr
    r = run_cli(mode, "--eval-data", "e.bin")
    assert r.returncode != 0 and "requires --safetensors and --eval-data" in r.stderr


def test_missing_data_file_is_reported(tmp_path):
    r = run_cli(*TRAIN[:1], "m", "--domain-data", str(tmp_path / "nope.bin"), "--ood-data", "o.bin",
                "--output", str(tmp_path / "ck.graft"), "--batch-size", "2")
    assert r.returncode != 0 and "Error" in r.stderr


def test_safetensors_tensor_info(tmp_path):
    import ctypes as C
    p = tmp_path / "a.safetensors"
    write_safetensors(str(p), {"x.weight": np.zeros((3, 5), np.float32), "n": np.ones(7, np.float32)},
                      {"n": "F32"})
    found, nd = C.c_int(), C.c_int()
    shape = (C.c_int64 * 8)()
    _lib.check(_lib.lib.glt_safetensors_tensor_info(str(p).encode(), b"x.weight", C.byref(found), shape,
                                                    C.byref(nd)))
    assert found.value == 1 and nd.value == 2 and list(shape[:2]) == [3, 5]
    _lib.check(_lib.lib.glt_safetensors_tensor_info(str(tmp_path).encode(), b"n", C.byref(found), shape,
                                                    C.byref(nd)))
    assert found.value == 1 and nd.value == 1 and shape[0] == 7
    _lib.check(_lib.lib.glt_safetensors_tensor_info(str(p).encode(), b"lm_head.weight", C.byref(found),
                                                    shape, C.byref(nd)))
    assert found.value == 0
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{\"x\": {\"dtype\"")
    with pytest.raises(_lib.GltError):
        _lib.check(_lib.lib.glt_safetensors_tensor_info(str(bad).encode(), b"x", C.byref(found), shape,
                                                        C.byref(nd)))


def test_train_state_flag_refusals(tmp_path):
    r = run_cli("--eval-only", "--safetensors", "m", "--eval-data", "e.bin", "--save-state", "x.state")
    assert r.returncode != 0 and "training-only" in r.stderr
    r = run_cli(*TRAIN, "--resume-state", "x.state", "--checkpoint", "c.graft")
    assert r.returncode != 0 and "incompatible with --checkpoint" in r.stderr
    r = run_cli(*TRAIN, "--resume-state", str(tmp_path / "none.state"))
    assert r.returncode != 0 and "does not exist" in r.stderr
    r = run_cli(*TRAIN, "--save-state", str(tmp_path))
    assert r.returncode != 0 and "--save-state path" in r.stderr
    r = run_cli("--help")
    assert "--resume-state" in r.stdout
