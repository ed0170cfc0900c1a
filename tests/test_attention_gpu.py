"""Fused attention: the tensor-core kernel (D = 64) and the CUDA-core one.

The fused op's definition is the five-op chain of hexlib/models/vit.py:183-190
(scale, transpose_hd, matmul, softmax, matmul). The chain rounds its scores
and probabilities to fp16 between ops; the fused kernel does not, so the bar
is set against the EXACT result of the chain's mathematics (float64 from the
same fp16 inputs, rounded once to fp16): within max-abs 2e-3 or one fp16
step. The unfused chain is checked to sit no closer to that exact result than
the kernel does, and whole plans with the rewrite are checked end to end.
"""
from __future__ import annotations

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan
from hexlib_b200.session import Session
from oracle import executor
from tests import gpu_util as U
from tests.tolerance import assert_close_f16

pytestmark = pytest.mark.gpu


def exact_attention(q, k, v, scale):
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    s = (q * scale) @ k.transpose(0, 2, 1)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return (p @ v).astype(np.float16).astype(np.float64)


def run_kernel(q, k, v, scale):
    Bn, T, D = q.shape
    dq, dk, dv = U.dev(q), U.dev(k), U.dev(v)
    y = U.empty((Bn, T, D), np.float16)
    U.call("hexlib_b200_attention_fp16", U.ptr(dq), U.ptr(dk), U.ptr(dv), U.ptr(y),
           Bn, T, D, float(scale), U.stream())
    return U.host(y)


@pytest.mark.parametrize("Bn,T,D,amp", [
    (12, 256, 64, 1.0),      # the 256^2 encoder's heads
    (4, 1024, 64, 1.0),      # 512^2
    (2, 4096, 64, 0.5),      # 1024^2: 32 key blocks, 16 query pairs
    (3, 200, 64, 1.0),       # partial query and key tiles
    (2, 100, 64, 2.0),       # one partial tile, larger logits
    (5, 300, 64, 1.0),
    (2, 64, 16, 1.0),        # tiny-config head dim: CUDA-core kernel
    (2, 130, 128, 1.0),      # wide heads: CUDA-core kernel
    (160, 512, 64, 1.0),     # 320 work items: every CTA walks two or three
    (300, 300, 64, 1.0),     # 600 items with ragged query and key tiles
])
def test_attention_matches_exact_math(Bn, T, D, amp):
    rng = np.random.default_rng(Bn * 1000 + T)
    q, k, v = ((rng.standard_normal((Bn, T, D)) * amp).astype(np.float16) for _ in range(3))
    scale = D ** -0.5
    got = run_kernel(q, k, v, scale)
    ref = exact_attention(q, k, v, scale)
    assert_close_f16(got, ref, what=f"attention {Bn}x{T}x{D}")


def test_attention_is_no_further_from_exact_than_the_unfused_chain():
    rng = np.random.default_rng(7)
    Bn, T, D = 6, 256, 64
    q, k, v = (rng.standard_normal((Bn, T, D)).astype(np.float16) for _ in range(3))
    got = run_kernel(q, k, v, 0.125).astype(np.float64)
    ref = exact_attention(q, k, v, 0.125)
    chain = executor.attention_chain(*(x.astype(np.float32) for x in (q, k, v)), 0.125)
    assert np.abs(got - ref).max() <= np.abs(chain - ref).max() + 1e-3


def test_attention_rows_sum_like_a_softmax():
    # v = all ones: every output row must be exactly the average of ones.
    Bn, T, D = 2, 384, 64
    rng = np.random.default_rng(3)
    q, k = (rng.standard_normal((Bn, T, D)).astype(np.float16) for _ in range(2))
    v = np.ones((Bn, T, D), np.float16)
    got = run_kernel(q, k, v, 0.125)
    assert np.abs(got.astype(np.float64) - 1.0).max() <= 1e-3


def test_fused_encoder_matches_the_oracle_at_256():
    cfg = G.qwen35_at(256)
    g = G.build_vision_encoder(cfg)
    w = F.weights(cfg, 0, g)
    imgs = F.images(cfg, 2, 11)
    fused = G.compile_for_cuda(g, attention=True, residual=True)
    plan = wholeplan.build_cuda_plan(fused, w, alias=True)
    assert plan.kinds.count("attention") == 12
    with Session(0) as s:
        s.load(plan, max_images=2)
        out = s.run(np.ascontiguousarray(imgs))
    for i in range(2):
        ref = executor.run(G.compile_for_cuda(g), dict(w, image=imgs[i]))["merger.out"]
        err = np.abs(out[i].astype(np.float64) - ref).max() / np.abs(ref).max()
        assert err < 1e-2, f"image {i}: relative error {err:.3e}"
