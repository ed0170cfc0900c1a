"""Plan replay on the CPU with the reference interpreter's storage semantics.

Restates hexlib/exec/interpreter.py:80-205 for what decides the numbers:
every graph input and const enters in the compute dtype (:111-132), every op
runs on compute-dtype arrays (:344-399), and every result is rounded to its
tensor's declared storage dtype when it is stored and read back as float32
(vtcm.py:90-127). The VTCM byte image, the DMA bookkeeping and the traffic
counters of the reference change no value, so they are not restated.

`backends` plays the role of the interpreter's per-kind hook (:134-150): a
mapping from op kind to a callable `(arrays, attrs) -> tuple of arrays` that
replaces the reference for that kind.
"""
from __future__ import annotations

from typing import Any, Callable, Mapping

import numpy as np

from oracle import ops

Backend = Callable[[tuple, Mapping[str, Any]], tuple]


def _graph_and_order(model):
    """Accept a graph (ops in order) or a compiled pair (ops in plan order)."""
    if hasattr(model, "plan") and hasattr(model, "graph"):
        graph = model.graph
        order = [s.op for s in model.plan.steps if getattr(s, "op", None) is not None]
        return graph, order
    return model, list(model.ops)


def run(model, feeds: Mapping[str, np.ndarray],
        backends: Mapping[str, Backend] | None = None) -> dict[str, np.ndarray]:
    graph, order = _graph_and_order(model)
    tensors = graph.tensors
    env: dict[str, np.ndarray] = {}
    required = list(graph.inputs) + [n for n, t in tensors.items() if t.const]
    for name in required:
        if name not in feeds:
            raise KeyError(f"missing feed for {name!r}")
        t = tensors[name]
        a = np.asarray(feeds[name])
        if tuple(a.shape) != tuple(t.shape):
            raise ValueError(f"feed {name!r} has shape {a.shape}, declared {t.shape}")
        env[name] = ops.store(a, t.dtype)
    for op in order:
        arrays = tuple(env[n] for n in op.inputs)
        fn = (backends or {}).get(op.kind) or ops.reference(op.kind)
        results = fn(arrays, dict(op.attrs))
        if not isinstance(results, tuple) or len(results) != len(op.outputs):
            raise ValueError(f"op {op.id} ({op.kind}) returned {type(results)}")
        for name, value in zip(op.outputs, results):
            t = tensors[name]
            value = np.asarray(value)
            if tuple(value.shape) != tuple(t.shape):
                raise ValueError(
                    f"op {op.id} ({op.kind}) wrote {name!r} with shape "
                    f"{value.shape}, declared {t.shape}")
            env[name] = ops.store(value, t.dtype)
    return {n: env[n] for n in graph.outputs}


# ---- composites: what a fused CUDA kind replaces, op by op ---------------------

def attention_chain(q, k, v, scale, dtype="fp16"):
    """The five-op chain hexlib/models/vit.py:183-190 writes for one block,
    q, k, v [Bn, T, D] in their [H, T, D] layout: scale -> transpose_hd ->
    matmul -> softmax -> matmul, with storage rounding after each op."""
    st = lambda x: ops.store(x, dtype)  # noqa: E731
    qs = st(ops.scale((q,), {"factor": scale})[0])
    kt = st(ops.transpose((k,), {"perm": (0, 2, 1)})[0])
    s = st(ops.matmul((qs, kt), {})[0])
    p = st(ops.softmax((s,), {"axis": -1})[0])
    return st(ops.matmul((p, v), {})[0])


def matmul_epilogue_residual_chain(a, w, bias, r, act="none", dtype="fp16"):
    """matmul_epilogue then the residual add(r, mm) that consumes it
    (vit.py:196, :203), rounded after each."""
    mm = ops.store(ops.matmul_epilogue((a, w, bias), {"act": act})[0], dtype)
    return ops.store(ops.add((r, mm), {})[0], dtype)
