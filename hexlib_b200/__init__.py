"""hexlib_b200 -- a B200 (sm_100a) execution backend for hexlib's plan executor.

The compute path is libhexlib_b200.so (hand-written CUDA for sm_100a behind a
C ABI, include/hexlib_b200.h). This package is the host side of it, written
as a mirror of the reference's own interfaces for the same path:

  wire        the batch blob and response (hexlib/runtime/wire.py)
  runner      KIND_ID, the CUDA variants' specs and `select`
              (hexlib/exec/runner.py, hexlib/runtime/genentry.py)
  graph       the IR, the Qwen3.5 vision-encoder builder and the fusion pass
              the plan executor consumes (hexlib/graph, hexlib/models)
  wholeplan   whole plan -> one blob over a const and a per-image arena
              (hexlib/exec/wholeplan.py), for B images at once
  session     a device session: stage weights, run images, read embeddings
  backends    per-op `interpreter_backends` (hexlib/exec/dsp.py:656-715)
  dist        image sharding over GPUs with one NCCL all-gather
"""
from __future__ import annotations

__all__ = ["__version__"]
__version__ = "0.1.0"
