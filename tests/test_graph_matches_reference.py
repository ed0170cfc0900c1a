"""The restated builder and fusion pass produce the reference's post-fusion
graph, op for op, at every configuration the benchmark uses; the CUDA-only
rewrites are checked for what they replace."""
from __future__ import annotations

import dataclasses
import json
import os
from collections import Counter

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PLANS = json.load(open(os.path.join(GOLDEN, "plans.json")))

TINY16 = G.VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                     patch_size=4, temporal_patch_size=2, in_channels=3,
                     spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                     rope_theta=10000.0, image_size=32, act_dtype="fp16",
                     weight_dtype="fp16")

CONFIGS = {
    "tiny_fp16": TINY16,
    "qwen35_256": G.qwen35_at(256),
    "qwen35_512": G.qwen35_at(512),
    "qwen35_1024": G.qwen35_at(1024),
}


def _norm_attrs(a):
    return {k: (list(v) if isinstance(v, tuple) else v) for k, v in dict(a).items()}


@pytest.mark.parametrize("key", sorted(CONFIGS))
def test_post_fusion_graph_equals_the_references(key):
    ref = PLANS[key]
    ep = G.compile_for_cuda(G.build_vision_encoder(CONFIGS[key]))
    g = ep.graph
    assert {n: [t.dtype, list(t.shape), t.const] for n, t in g.tensors.items()} == ref["tensors"]
    mine = {o.id: [o.id, o.kind, list(o.inputs), list(o.outputs), _norm_attrs(o.attrs)]
            for o in g.ops}
    theirs = {o[0]: o for o in ref["ops"]}
    assert mine == theirs
    assert list(g.inputs) == ref["inputs"] and list(g.outputs) == ref["outputs"]
    assert len(g.ops) == ref["n_steps"]


def test_reference_plan_json_loads_in_plan_order():
    text = open(os.path.join(GOLDEN, "tiny_compiled.json")).read()
    ep = G.from_compiled_json(text)
    assert [o.id for o in ep.graph.ops] == PLANS["tiny_fp16"]["step_order"]
    assert [s.op.id for s in ep.plan.steps] == PLANS["tiny_fp16"]["step_order"]


def test_the_references_256_json_plan_is_our_256_plan():
    """The reference's compiled.to_json artefact of its 256^2 plan loads into
    the same graph this module builds, in the reference's step order."""
    import gzip
    with gzip.open(os.path.join(GOLDEN, "qwen35_256_compiled.json.gz"), "rt") as fh:
        ep = G.from_compiled_json(fh.read())
    ours = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256))).graph
    assert [o.id for o in ep.graph.ops] == PLANS["qwen35_256"]["step_order"]
    assert {n: (t.dtype, t.shape, t.const) for n, t in ep.graph.tensors.items()} == \
        {n: (t.dtype, t.shape, t.const) for n, t in ours.tensors.items()}
    by_id = {o.id: o for o in ours.ops}
    for o in ep.graph.ops:
        mine = by_id[o.id]
        assert (o.kind, o.inputs, o.outputs) == (mine.kind, mine.inputs, mine.outputs)
        assert _norm_attrs(o.attrs) == _norm_attrs(mine.attrs)
    assert ep.graph.problems() == []


def test_encoder_op_census_at_256():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)))
    c = Counter(o.kind for o in ep.graph.ops)
    assert c == Counter({"matmul_epilogue": 75, "transpose": 60, "reshape": 49, "add": 25,
                         "layernorm": 25, "rope_2d": 24, "matmul": 24, "scale": 12,
                         "softmax": 12, "patchify": 1, "cast": 1})


def test_attention_rewrite_replaces_exactly_the_five_op_chain():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)), attention=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["attention"] == 12
    assert c["softmax"] == 0 and c["matmul"] == 0 and c["scale"] == 0
    assert c["transpose"] == 48          # the perm (0,2,1) transposes are gone
    for o in ep.graph.ops:
        if o.kind == "attention":
            assert o.attrs["scale"] == 0.125
            assert all(ep.graph.tensors[n].shape == (12, 256, 64) for n in o.inputs)
    assert not any(n.endswith(".scores") or n.endswith(".probs") for n in ep.graph.tensors)


def test_residual_rewrite_folds_the_24_residual_adds():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)), residual=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["matmul_epilogue_residual"] == 24
    assert c["add"] == 1                 # only the pos_embed add remains
    for o in ep.graph.ops:
        if o.kind == "matmul_epilogue_residual":
            assert o.attrs["act"] == "none"
            assert not ep.graph.tensors[o.inputs[3]].const


def test_rewrites_apply_to_a_reference_compiled_pair():
    text = open(os.path.join(GOLDEN, "tiny_compiled.json")).read()
    ep = G.from_compiled_json(text)
    rw = G.rewrite_compiled(ep, attention=True, residual=True)
    c = Counter(o.kind for o in rw.graph.ops)
    assert c["attention"] == 2 and c["matmul_epilogue_residual"] == 4
    assert rw.graph.problems() == []


def test_rope_epilogue_rewrite_moves_the_rotation_into_the_qkv_gemm():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)), residual=True, qkv=True,
                            rope_epilogue=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["matmul_epilogue_rope"] == 12 and c["attention_qkv"] == 12
    assert c["rope_qk"] == 0 and c["rope_2d"] == 0 and c["transpose"] == 0
    assert c["matmul_epilogue"] == 12 + 3
    # 12 concatenated weights and biases, one set of segment tables for all blocks
    assert len(ep.derived) == 24 + 3
    for o in ep.graph.ops:
        if o.kind == "matmul_epilogue_rope":
            assert o.attrs == {"act": "none", "rope_cols": 2 * 12 * 64}
            assert ep.graph.tensors[o.outputs[0]].shape == (256, 3, 12, 64)
            segs = [ep.graph.tensors[n] for n in o.inputs[3:]]
            assert [(t.dtype, t.shape) for t in segs] == [
                ("fp32", (512, 16)), ("fp32", (512, 16)), ("int32", (256, 2))]
            assert all(ep.derived[n][0] == "rope_segments" for n in o.inputs[3:])
    assert ep.graph.problems() == []
    # a quantized weight takes the same epilogue (the GEMM reads the session's
    # fp16 copy of it), its packed weight staying q4_0 on the wire
    q = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256, weight_dtype="q4_0")),
                           residual=True, qkv=True, rope_epilogue=True)
    cq = Counter(o.kind for o in q.graph.ops)
    assert cq["rope_qk"] == 0 and cq["matmul_epilogue_rope"] == 12
    for o in q.graph.ops:
        if o.kind == "matmul_epilogue_rope":
            assert q.graph.tensors[o.inputs[1]].dtype == "q4_0"


def test_layernorm_fold_rewrites_every_layernorm_that_feeds_a_gemm():
    g = G.build_vision_encoder(G.qwen35_at(256))
    ep = G.compile_for_cuda(g, residual=True, qkv=True, rope_epilogue=True, ln_fold=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["ln_stats"] == 24 and c["matmul_epilogue_ln_rope"] == 12
    assert c["matmul_epilogue_ln"] == 12
    # the merger's layernorm feeds a reshape, not a GEMM: it stays
    assert c["layernorm"] == 1
    assert ep.graph.problems() == []
    for o in ep.graph.ops:
        if o.kind == "matmul_epilogue_ln":
            x, wf, cols, stats = o.inputs
            t = ep.graph.tensors
            assert t[wf].dtype == "fp16" and t[cols].shape == (2, t[wf].shape[1])
            assert t[stats].shape == (256, 2) and not t[stats].const
            assert ep.derived[wf][0] == "ln_fold_w" and ep.derived[cols][0] == "ln_fold_cols"
        if o.kind == "matmul_epilogue_ln_rope":
            segtab = ep.graph.tensors[o.inputs[4]]
            assert segtab.shape == (512, 2, 16) and segtab.dtype == "fp32"
    # quantized weights are not folded (the fold would requantize them)
    q = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256, weight_dtype="q4_0")),
                           residual=True, qkv=True, rope_epilogue=True, ln_fold=True)
    assert Counter(o.kind for o in q.graph.ops)["ln_stats"] == 0


def test_patchify_cast_rewrite_replaces_the_pair():
    g = G.build_vision_encoder(G.qwen35_at(256))
    ep = G.compile_for_cuda(g, residual=True, patch_cast=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["patchify_cast"] == 1 and c["patchify"] == 0 and c["cast"] == 0
    op = next(o for o in ep.graph.ops if o.kind == "patchify_cast")
    assert ep.graph.tensors[op.outputs[0]].dtype == "fp16"
    assert ep.graph.problems() == []


def test_the_fold_identity_holds_in_float64():
    """rstd (x @ W' - mean colsum(W')) + (beta @ W + b) is layernorm(x) @ W + b
    up to the one fp16 rounding of W' = diag(gamma) W."""
    r = np.random.default_rng(0)
    K, N = 64, 32
    x = (r.standard_normal((5, K)) + 4.0).astype(np.float16).astype(np.float64)
    gamma = (1 + 0.1 * r.standard_normal(K)).astype(np.float32)
    beta = (0.1 * r.standard_normal(K)).astype(np.float32)
    w = (0.05 * r.standard_normal((K, N))).astype(np.float16)
    b = (0.02 * r.standard_normal(N)).astype(np.float32)
    mean = x.mean(1, keepdims=True)
    rstd = 1 / np.sqrt(((x - mean) ** 2).mean(1, keepdims=True) + 1e-6)
    exact = ((x - mean) * rstd * gamma + beta) @ w.astype(np.float64) + b
    wf = wholeplan.ln_fold_w(gamma, w).astype(np.float64)
    cols = wholeplan.ln_fold_cols(gamma, beta, w, b).astype(np.float64)
    folded = rstd * (x @ wf - mean * cols[1]) + cols[0]
    assert np.abs(folded - exact).max() < 4e-3 * np.abs(exact).max()


def test_rope_segments_rebuild_the_tables_exactly():
    cfg = G.qwen35_at(512)
    w = F.weights(cfg, 0, G.build_vision_encoder(cfg))
    cos, sin = w["rope_cos"], w["rope_sin"]
    seg_cos, seg_sin, idx = wholeplan.rope_segments(cos, sin)
    T = cos.shape[0]
    assert idx.dtype == np.int32 and idx.shape == (T, 2) and seg_cos.shape == (2 * T, 16)
    half = seg_cos[idx].reshape(T, 32)
    np.testing.assert_array_equal(np.concatenate([half, half], 1), cos)
    half = seg_sin[idx].reshape(T, 32)
    np.testing.assert_array_equal(np.concatenate([half, half], 1), sin)
    # a 32 x 32 grid repeats each segment along a row or a column of patches
    assert idx.max() + 1 <= 64
    ang = np.random.default_rng(0).uniform(-3, 3, (50, 32)).astype(np.float32)
    ang = np.concatenate([ang, ang], 1)
    sc, ss, ix = wholeplan.rope_segments(np.cos(ang), np.sin(ang))
    np.testing.assert_array_equal(sc[ix].reshape(50, 32), np.cos(ang)[:, :32])
    with pytest.raises(wholeplan.WholePlanError):
        wholeplan.rope_segments(np.zeros((4, 32), np.float32), np.zeros((4, 32), np.float32))
    ang[3, 40] += 1.0                       # no longer half-symmetric
    with pytest.raises(wholeplan.WholePlanError):
        wholeplan.rope_segments(np.cos(ang), np.sin(ang))


def test_invalid_configs_are_refused():
    with pytest.raises(ValueError):
        G.build_vision_encoder(dataclasses.replace(TINY16, image_size=30))
    with pytest.raises(ValueError):
        G.build_vision_encoder(dataclasses.replace(TINY16, num_heads=5))


def test_qkv_rewrite_packs_the_projections_and_drops_the_transposes():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)), residual=True, qkv=True)
    c = Counter(o.kind for o in ep.graph.ops)
    assert c["rope_qk"] == 12 and c["attention_qkv"] == 12
    assert c["transpose"] == 0 and c["rope_2d"] == 0 and c["attention"] == 0
    # qkv and fc1 per block; patch embed, merger fc1/fc2
    assert c["matmul_epilogue"] == 12 + 12 + 3
    assert len(ep.derived) == 24
    for o in ep.graph.ops:
        if o.kind == "matmul_epilogue" and ep.graph.tensors[o.inputs[1]].shape == (768, 2304):
            how, parts, axis = ep.derived[o.inputs[1]]
            assert how == "concat" and axis == 1 and len(parts) == 3
            assert ep.graph.tensors[o.outputs[0]].shape == (256, 3, 12, 64)
        if o.kind == "rope_qk":
            assert ep.graph.tensors[o.outputs[0]].shape == (256, 3, 12, 64)
        if o.kind == "attention_qkv":
            assert ep.graph.tensors[o.outputs[0]].shape == (256, 12, 64)
    assert ep.graph.problems() == []
