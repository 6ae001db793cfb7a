"""CPU oracle for the grafted-MLP hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference (Hinedes/GLT) algorithm on the CPU so
the CUDA library can be checked against it:
  bitexact.py   bf16 bias-trick rounding, shadow bake, GRFT checkpoint bytes,
                .bin loader, splitmix64 batch walk, LR schedule (numpy)
  graft_ops.py  the six graft GEMMs in the reference's operand orientations
  ref_math.py   fp32 decoder forward / recompute / backward / loss / clip /
                AdamW in overlay and concat geometry (torch, CPU)

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
its --impl reference arm) may import it, and only as the checker or the
timed CPU baseline -- never as the product path.  Parity is pinned against
the reference's own golden vectors (tests/golden/reference_kats.json).
"""
