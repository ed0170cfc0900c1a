"""The numpy oracle against the reference's own C baselines (kernels/*/
baseline.c compiled into oracle/_ref), at the benchmark's per-kernel gate
shapes: two independent statements of each kernel must agree."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import cref, ops
from tests.tolerance import assert_bit_exact, assert_close_f16

pytestmark = pytest.mark.skipif(not cref.available(),
                                reason="oracle/_ref not built (python oracle/build_ref.py)")

F = ctypes.c_float


def r16(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float16)


def o16(kind, arrays, attrs):
    (out,) = ops.reference(kind)(tuple(np.asarray(a, np.float32) for a in arrays), attrs)
    return ops.store(out, "fp16").astype(np.float16)


def test_add():
    n = 256 * 768 + 4
    a, b, y = r16(n, 1), r16(n, 2), np.empty(n, np.float16)
    cref.call("add_fp16", a, b, y, n)
    assert_bit_exact(y, o16("add", (a, b), {}), "add")


def test_scale():
    n = 4100
    x, y = r16(n, 3), np.empty(n, np.float16)
    cref.call("scale_fp16", x, y, n, F(0.125))
    assert_bit_exact(y, o16("scale", (x,), {"factor": 0.125}), "scale")


def test_cast():
    n = 4133
    x = (np.random.default_rng(4).standard_normal(n) * 50).astype(np.float32)
    y = np.empty(n, np.float16)
    cref.call("cast_f32_f16", x, y, n)
    assert_bit_exact(y, x.astype(np.float16), "cast")


def test_layernorm():
    R, C = 256, 768
    x = r16((R, C), 5)
    w = (1 + np.random.default_rng(6).standard_normal(C) * 0.02).astype(np.float32)
    b = (np.random.default_rng(7).standard_normal(C) * 0.02).astype(np.float32)
    y = np.empty((R, C), np.float16)
    cref.call("layernorm_fp16", x, w, b, y, R, C, F(1e-6))
    assert_close_f16(y, o16("layernorm", (x, w, b), {"eps": 1e-6}), what="layernorm")


def test_rmsnorm():
    R, C = 256, 768
    x, w = r16((R, C), 8), r16(C, 9, 0.5)
    y = np.empty((R, C), np.float16)
    cref.call("rmsnorm_fp16", x, w, y, R, C, F(1e-5))
    assert_close_f16(y, o16("rmsnorm", (x, w), {"eps": 1e-5}), what="rmsnorm")


def test_softmax():
    R, C = 12 * 256, 256
    x = r16((R, C), 10, 3.0)
    x[0, 3] = 90.0
    y = np.empty((R, C), np.float16)
    cref.call("softmax_fp16", x, y, R, C)
    assert_close_f16(y, o16("softmax", (x,), {"axis": -1}), what="softmax")


def test_rope():
    T, H, D = 256, 12, 64
    x = r16((T, H, D), 11)
    ang = np.random.default_rng(12).uniform(-3, 3, (T, D)).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    y = np.empty((T, H, D), np.float16)
    cref.call("rope_2d_fp16", x, c, s, y, T, H, D)
    assert_close_f16(y, o16("rope_2d", (x, c, s), {}), what="rope")


def test_transposes():
    T, H, D = 256, 12, 64
    x, y = r16((T, H, D), 13), np.empty((H, T, D), np.float16)
    cref.call("transpose_th_fp16", x, y, T, H, D)
    assert_bit_exact(y, np.ascontiguousarray(x.transpose(1, 0, 2)), "transpose_th")
    B, T, D = 12, 256, 64
    x, y = r16((B, T, D), 14), np.empty((B, D, T), np.float16)
    cref.call("transpose_hd_fp16", x, y, B, T, D)
    assert_bit_exact(y, np.ascontiguousarray(x.transpose(0, 2, 1)), "transpose_hd")


def test_patchify():
    img = np.random.default_rng(15).standard_normal((3, 2, 256, 256)).astype(np.float32)
    y = np.empty((256, 1536), np.float32)
    cref.call("patchify_fp32", img, y, 3, 2, 256, 256, 16, 2, 16, 16)
    attrs = {"patch": 16, "temporal_patch": 2, "merge": 2, "grid_h": 16, "grid_w": 16}
    assert_bit_exact(y, ops.patchify((img,), attrs)[0], "patchify")


def test_matmul():
    Bn, M, K, N = 12, 256, 64, 256
    a, b = r16((Bn, M, K), 16), r16((Bn, K, N), 17, 0.125)
    y = np.empty((Bn, M, N), np.float16)
    cref.call("matmul_fp16", a, b, y, Bn, M, K, N)
    assert_close_f16(y, o16("matmul", (a, b), {}), what="matmul")


@pytest.mark.parametrize("M,K,N,act", [(256, 768, 768, 0), (64, 768, 3072, 1), (8, 96, 64, 2)])
def test_quantized_matmul_epilogue(M, K, N, act):
    """The reference's only matmul_epilogue kernel takes a q4_0 weight
    (baseline.c:49-97); the oracle's dequantize-to-fp16 statement of it must
    agree, on weights packed by this repository's own quantizer."""
    from hexlib_b200 import quant
    from oracle import quant as oq
    a = r16((M, K), 40)
    w = (np.random.default_rng(41).standard_normal((K, N)) * 0.05).astype(np.float32)
    bias = (np.random.default_rng(42).standard_normal(N) * 0.02).astype(np.float32)
    raw = np.frombuffer(quant.quantize_q4_0(w), np.uint8).copy()
    got = np.zeros((M, N), np.float16)
    cref.call("matmul_epilogue_fp16", a, raw, bias, got, M, K, N, act)
    act_name = {0: "none", 1: "gelu_tanh", 2: "gelu_erf"}[act]
    want = oq.matmul_epilogue_quant(a, raw.tobytes(), bias, K, N, "q4_0", act_name)
    assert_close_f16(got, ops.store(want, "fp16").astype(np.float16), what=f"q4_0 {act_name}")
