"""Host-side helpers of bench.py (no GPU): the NCCL log summary.

NCCL's TUNING lines name the all-reduce algorithm and protocol by index in
older releases and by name in 2.2x; both forms must land in the bench
line's `nccl.allreduce` table, one entry per message size with its call
count.
"""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_nccl_summary_both_log_forms(tmp_path):
    log = tmp_path / "nccl.log"
    log.write_text(
        "vm:1:1 [0] NCCL INFO NCCL version 2.28.9+cuda12.9\n"
        "vm:1:1 [0] NCCL INFO AllReduce: 201326592 Bytes -> Algo RING proto SIMPLE channel{Lo..Hi}={0..31}\n"
        "vm:1:1 [0] NCCL INFO AllReduce: 201326592 Bytes -> Algo RING proto SIMPLE channel{Lo..Hi}={0..31}\n"
        "vm:1:1 [0] NCCL INFO AllReduce: 4096 Bytes -> Algo 4 proto 0 channel{Lo..Hi}={0..3}\n"
        "vm:1:1 [0] NCCL INFO NVLS multicast support is available on dev 0 (NVLS_NCHANNELS 24)\n")
    s = _bench().nccl_summary(str(log))
    assert s["version"] == "NCCL version 2.28.9+cuda12.9"
    assert s["allreduce"]["201326592 B"] == {"algo": "RING", "proto": "SIMPLE", "calls": 2}
    assert s["allreduce"]["4096 B"] == {"algo": "NVLS", "proto": "LL", "calls": 1}
    assert s["nvls_lines"]


def test_nccl_summary_missing_log(tmp_path):
    assert _bench().nccl_summary(str(tmp_path / "absent.log")) == {"log": "unavailable"}
