"""oracle -- TEST INFRASTRUCTURE ONLY: the CPU checker for hexlib_b200.

A numpy restatement of the reference's arithmetic for the plan-executor path
(hexlib/graph/opdefs/*.py and hexlib/exec/interpreter.py + vtcm.py), plus a
recipe that compiles the reference's own scalar kernels/*/baseline.c into
oracle/_ref/ as a second, independent checker.

Pinned by tests/test_oracle_pinning.py against golden vectors produced by the
reference itself (tests/golden/make_golden.py, run where the reference is
importable): the transformers-generated tiny-encoder golden
(hexlib/tests/data/qwen35_vision_tiny.npz), the reference interpreter's own
fp32 and fp16 plan replays, and per-op outputs of the reference op registry.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package, and only to check or to time the reference algorithm -- never
as the thing measured or shipped. Nothing in hexlib_b200/ imports it.
"""
