"""The per-op plug-in path: the interpreter's backend hook served by CUDA
kernels, one op at a time, exactly as hexlib's interpreter.run(...,
backends=...) would call them."""
from __future__ import annotations

import os

import numpy as np
import pytest

from hexlib_b200 import backends
from hexlib_b200 import graph as G
from oracle import executor

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY16 = G.VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                     patch_size=4, temporal_patch_size=2, in_channels=3,
                     spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                     rope_theta=10000.0, image_size=32, act_dtype="fp16",
                     weight_dtype="fp16")


def test_every_compute_op_runs_on_the_gpu_and_the_answer_holds():
    z = np.load(os.path.join(GOLDEN, "tiny.npz"))
    f = {k[6:]: z[k] for k in z.files if k.startswith("feed::")}
    ep = G.compile_for_cuda(G.build_vision_encoder(TINY16))
    be = backends.interpreter_backends()
    calls: dict[str, int] = {}

    def counted(kind, fn):
        def run(arrays, attrs):
            calls[kind] = calls.get(kind, 0) + 1
            return fn(arrays, attrs)
        return run

    hooked = {k: counted(k, v) for k, v in be.items()}
    got = executor.run(ep, f, backends=hooked)["merger.out"]
    ref = executor.run(ep, f)["merger.out"]
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-2
    kinds = {o.kind for o in ep.graph.ops} - {"reshape"}
    assert set(calls) == kinds
    assert np.abs(got - z["interp_fp16_fp16"]).max() / np.abs(z["interp_fp16_fp16"]).max() < 1e-2


def test_backend_refuses_a_variant_no_kernel_serves():
    be = backends.interpreter_backends(["transpose", "softmax"])
    x = np.zeros((2, 3, 4), np.float32)
    with pytest.raises(ValueError):
        be["transpose"]((x,), {"perm": (2, 1, 0)})
    with pytest.raises(ValueError):
        be["softmax"]((x,), {"axis": 0})
