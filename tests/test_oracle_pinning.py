"""The oracle is pinned before it is trusted.

Against fixtures the reference produced (tests/golden/make_golden.py): the
transformers golden of the tiny encoder, the reference interpreter's own fp32
and fp16 plan replays, and the op registry's outputs for every op kind.
"""
from __future__ import annotations

import dataclasses
import json
import os

import numpy as np
import pytest

from hexlib_b200 import graph as G
from oracle import executor, ops

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

TINY = G.VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                   patch_size=4, temporal_patch_size=2, in_channels=3,
                   spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                   rope_theta=10000.0, image_size=32, act_dtype="fp32",
                   weight_dtype="fp32")


def tiny_feeds():
    z = np.load(os.path.join(GOLDEN, "tiny.npz"))
    return {k[len("feed::"):]: z[k] for k in z.files if k.startswith("feed::")}, z


def test_tiny_fp32_matches_the_transformers_golden():
    feeds, z = tiny_feeds()
    g = G.build_vision_encoder(TINY)
    out = executor.run(G.compile_for_cuda(g), feeds)[g.outputs[0]]
    np.testing.assert_allclose(out, z["expected_merged"], rtol=1e-4, atol=1e-5)


def test_tiny_fp32_matches_the_reference_interpreter():
    feeds, z = tiny_feeds()
    g = G.build_vision_encoder(TINY)
    out = executor.run(G.compile_for_cuda(g), feeds)[g.outputs[0]]
    assert np.abs(out - z["interp_fp32_fp32"]).max() < 1e-6


def test_tiny_fp16_matches_the_reference_interpreter():
    feeds, z = tiny_feeds()
    cfg = dataclasses.replace(TINY, act_dtype="fp16", weight_dtype="fp16")
    g = G.build_vision_encoder(cfg)
    out = executor.run(G.compile_for_cuda(g), feeds)[g.outputs[0]]
    ref = z["interp_fp16_fp16"]
    # Same storage rounding at every op boundary; only float64-vs-float64
    # library differences remain, which flip at most an fp16 rounding.
    assert np.abs(out - ref).max() <= 2e-3
    assert np.mean(out == ref) > 0.9


def test_unfused_and_fused_graphs_agree_in_the_oracle():
    feeds, z = tiny_feeds()
    g = G.build_vision_encoder(TINY)
    a = executor.run(g, feeds)[g.outputs[0]]
    b = executor.run(G.compile_for_cuda(g), feeds)[g.outputs[0]]
    assert np.abs(a - b).max() < 1e-6


def test_a_wrong_epsilon_would_be_caught():
    feeds, z = tiny_feeds()
    g = G.build_vision_encoder(dataclasses.replace(TINY, layernorm_eps=1e-1))
    out = executor.run(g, feeds)[g.outputs[0]]
    assert not np.allclose(out, z["expected_merged"], rtol=1e-4, atol=1e-5)


def test_patchify_matches_upstreams_literal_permute_chain():
    feeds, z = tiny_feeds()
    attrs = {"patch": 4, "temporal_patch": 2, "merge": 2, "grid_h": 8, "grid_w": 8}
    got = ops.patchify((feeds["image"],), attrs)[0]
    np.testing.assert_array_equal(got, z["patches_upstream"])


def _op_cases():
    z = np.load(os.path.join(GOLDEN, "ops.npz"))
    meta = json.loads(bytes(z["__meta__"]).decode())
    for name, m in meta.items():
        arrays = tuple(z[f"{name}::in{i}"] for i in range(m["n_in"]))
        attrs = {k: (tuple(v) if isinstance(v, list) else v) for k, v in m["attrs"].items()}
        yield name, m["kind"], arrays, attrs, z[f"{name}::out"]


@pytest.mark.parametrize("case", list(_op_cases()), ids=lambda c: c[0])
def test_oracle_op_matches_the_registry(case):
    name, kind, arrays, attrs, want = case
    (got,) = ops.reference(kind)(arrays, attrs)
    assert got.shape == want.shape
    if kind in ("transpose", "patchify", "reshape", "cast", "add", "scale", "matmul",
                "matmul_epilogue", "rope_2d"):
        # same float32 arithmetic in the same order: identical
        tol = 0.0 if kind in ("transpose", "patchify", "reshape", "cast", "add", "scale",
                              "rope_2d") else 1e-6
        assert np.abs(got.astype(np.float64) - want).max() <= tol * max(1.0, np.abs(want).max())
    else:
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)


def test_rope_tables_match_the_reference_loader():
    from hexlib_b200 import feeds
    t = np.load(os.path.join(GOLDEN, "tables.npz"))
    for key, cfg in (("tiny", TINY), ("qwen35_256", G.qwen35_at(256))):
        c, s = feeds.rope_tables(cfg)
        np.testing.assert_array_equal(c, t[f"{key}::cos"])
        np.testing.assert_array_equal(s, t[f"{key}::sin"])


def test_fused_chains_are_the_ops_they_replace():
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal((2, 16, 8)).astype(np.float16).astype(np.float32)
               for _ in range(3))
    got = executor.attention_chain(q, k, v, 0.125)
    s = (q * 0.125).astype(np.float16).astype(np.float32) @ k.transpose(0, 2, 1)
    s = s.astype(np.float16).astype(np.float64)
    p = np.exp(s - s.max(-1, keepdims=True))
    p = (p / p.sum(-1, keepdims=True)).astype(np.float16).astype(np.float32)
    want = (p @ v).astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(got, want)
