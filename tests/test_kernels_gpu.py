"""Per-kernel parity: each C-ABI kernel entry against the oracle.

Shapes are the per-kernel gate shapes of the benchmark (fp16 ~N(0,1), seeded)
plus the edge cases the reference's own harnesses use: element counts with a
tail (4100, 4133), narrow rows (C=64, which is what exposes an unbiased
variance), non-multiple-of-vector widths, the softmax overflow row (a 90.0
that overflows exp in fp16) and the fp16-sum row, odd transposes (D=7, T=40),
and GEMM shapes that exercise the CUDA-core fallback (K or N not a multiple
of 8) next to the tensor-core path.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ops
from tests import gpu_util as G
from tests.tolerance import assert_bit_exact, assert_close_f16

pytestmark = pytest.mark.gpu


def rng(seed=0):
    return np.random.default_rng(seed)


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def randn16(shape, seed=0, scale=1.0):
    return f16(rng(seed).standard_normal(shape) * scale)


def oracle16(kind, arrays, attrs):
    """Oracle result rounded to fp16 storage, from fp16 inputs."""
    arrs = tuple(np.asarray(a, np.float32) for a in arrays)
    (out,) = ops.reference(kind)(arrs, attrs)
    return ops.store(out, "fp16")


# ---- elementwise ---------------------------------------------------------

@pytest.mark.parametrize("n", [256 * 768, 4100, 8, 1])
def test_add_fp16_is_bit_exact(n):
    a, b = randn16(n, 1), randn16(n, 2)
    y = G.empty(n, np.float16)
    da, db = G.dev(a), G.dev(b)
    G.call("hexlib_b200_add_fp16", G.ptr(da), G.ptr(db), G.ptr(y), n, G.stream())
    assert_bit_exact(G.host(y), f16(oracle16("add", (a, b), {})), "add")


@pytest.mark.parametrize("n", [256 * 768, 4100])
def test_add_fp16_f32_rounds_once(n):
    a = randn16(n, 3)
    b = rng(4).standard_normal(n).astype(np.float32) * 0.02
    y = G.empty(n, np.float16)
    da, db = G.dev(a), G.dev(b)
    G.call("hexlib_b200_add_fp16_f32", G.ptr(da), G.ptr(db), G.ptr(y), n, G.stream())
    want = f16(ops.add((a.astype(np.float32), b), {})[0])
    assert_bit_exact(G.host(y), want, "add fp16+fp32")


@pytest.mark.parametrize("n", [256 * 768, 4100])
def test_scale_by_an_eighth_is_bit_exact(n):
    x = randn16(n, 5)
    y = G.empty(n, np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_scale_fp16", G.ptr(dx), G.ptr(y), n, 0.125, G.stream())
    assert_bit_exact(G.host(y), f16(oracle16("scale", (x,), {"factor": 0.125})), "scale")


def test_scale_general_factor():
    n = 4100
    x = randn16(n, 6)
    y = G.empty(n, np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_scale_fp16", G.ptr(dx), G.ptr(y), n, 0.3, G.stream())
    want = f16(ops.scale((x.astype(np.float32),), {"factor": np.float32(0.3)})[0])
    assert_bit_exact(G.host(y), want, "scale 0.3")


@pytest.mark.parametrize("n", [256 * 768, 4160, 4133])
def test_cast_rounds_to_nearest_even(n):
    x = (rng(7).standard_normal(n) * 3).astype(np.float32)
    x[:4] = [65519.0, 65520.0, 1e-8, -2.0 ** -25]  # overflow edge, subnormals
    y = G.empty(n, np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_cast_f32_f16", G.ptr(dx), G.ptr(y), n, G.stream())
    assert_bit_exact(G.host(y), x.astype(np.float16), "cast")


# ---- rows -------------------------------------------------------------------

@pytest.mark.parametrize("R,C", [
    (256, 768), (4, 64), (3, 1000), (2, 256), (5, 1024),
    (4100, 64), (37, 128),            # 8 and 16 lanes per row, rows ending mid-warp
    (3, 2048), (5, 4096), (2, 8192),  # a CTA per row
    (4100, 768), (5000, 256), (4099, 512), (4096, 1024),  # many rows per warp, ragged end
])
def test_layernorm(R, C):
    x = randn16((R, C), 8)
    w = (1.0 + rng(9).standard_normal(C) * 0.02).astype(np.float32)
    b = (rng(10).standard_normal(C) * 0.02).astype(np.float32)
    y = G.empty((R, C), np.float16)
    dx, dw, db = G.dev(x), G.dev(w), G.dev(b)
    G.call("hexlib_b200_layernorm_fp16", G.ptr(dx), G.ptr(dw), G.ptr(db), G.ptr(y),
           R, C, 1e-6, G.stream())
    assert_close_f16(G.host(y), oracle16("layernorm", (x, w, b), {"eps": 1e-6}), what="layernorm")


def test_layernorm_distinguishes_biased_variance():
    # C=64 is where dividing by C-1 instead of C moves outputs by ~0.8%.
    R, C = 4, 64
    x = randn16((R, C), 11)
    w = np.ones(C, np.float32)
    b = np.zeros(C, np.float32)
    y = G.empty((R, C), np.float16)
    dx, dw, db = G.dev(x), G.dev(w), G.dev(b)
    G.call("hexlib_b200_layernorm_fp16", G.ptr(dx), G.ptr(dw), G.ptr(db), G.ptr(y),
           R, C, 1e-6, G.stream())
    got = G.host(y).astype(np.float64)
    xd = x.astype(np.float64)
    unbiased = (xd - xd.mean(-1, keepdims=True)) / np.sqrt(xd.var(-1, ddof=1, keepdims=True) + 1e-6)
    assert np.abs(got - unbiased).max() > 4e-3
    assert_close_f16(got, oracle16("layernorm", (x, w, b), {"eps": 1e-6}), what="layernorm C=64")


@pytest.mark.parametrize("R,C", [(256, 768), (8, 128), (3, 4096), (2, 100),
                                 (4100, 64), (3, 2048), (2, 8192)])
def test_rmsnorm(R, C):
    x = randn16((R, C), 12)
    w = f16(1.0 + rng(13).standard_normal(C) * 0.1)
    y = G.empty((R, C), np.float16)
    dx, dw = G.dev(x), G.dev(w)
    G.call("hexlib_b200_rmsnorm_fp16", G.ptr(dx), G.ptr(dw), G.ptr(y), R, C, 1e-5, G.stream())
    assert_close_f16(G.host(y), oracle16("rmsnorm", (x, w), {"eps": 1e-5}), what="rmsnorm")


@pytest.mark.parametrize("R,C", [(12 * 256, 256), (6, 256), (64, 1024), (4, 4096), (5, 1000),
                                 (3, 33), (4100, 64), (37, 128), (3, 2048), (2, 8192)])
def test_softmax(R, C):
    x = randn16((R, C), 14, scale=3.0)
    if R >= 2:
        x[0, 7] = 90.0          # exp(90) overflows fp16 and fp32 without the max shift
        x[1, :] = f16(np.linspace(-1, 1, C))  # a row whose fp16 running sum loses mass
    y = G.empty((R, C), np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_softmax_fp16", G.ptr(dx), G.ptr(y), R, C, G.stream())
    got = G.host(y)
    assert_close_f16(got, oracle16("softmax", (x,), {"axis": -1}), what="softmax")
    assert np.allclose(got.astype(np.float64).sum(-1), 1.0, atol=C * 2e-4)


@pytest.mark.parametrize("T,H,D", [(256, 12, 64), (6, 3, 64), (5, 2, 40), (4, 3, 6)])
def test_rope_2d(T, H, D):
    x = randn16((T, H, D), 15)
    ang = rng(16).uniform(-3, 3, (T, D)).astype(np.float32)  # halves differ on purpose
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    y = G.empty((T, H, D), np.float16)
    dx, dc, ds = G.dev(x), G.dev(cos), G.dev(sin)
    G.call("hexlib_b200_rope_2d_fp16", G.ptr(dx), G.ptr(dc), G.ptr(ds), G.ptr(y),
           T, H, D, G.stream())
    want = oracle16("rope_2d", (x, cos, sin), {})
    got = G.host(y)
    # fp32 products and sum rounded separately, as the registry does: bit-exact.
    assert_bit_exact(got, f16(want), "rope_2d")


# ---- movement -----------------------------------------------------------------

@pytest.mark.parametrize("T,H,D", [(256, 12, 64), (8, 3, 64), (8, 3, 40), (5, 3, 7), (1024, 12, 64)])
def test_transpose_th_is_bit_exact(T, H, D):
    x = randn16((T, H, D), 17)
    y = G.empty((H, T, D), np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_transpose_th_fp16", G.ptr(dx), G.ptr(y), T, H, D, G.stream())
    assert_bit_exact(G.host(y), np.ascontiguousarray(x.transpose(1, 0, 2)), "transpose_th")


@pytest.mark.parametrize("B,T,D", [
    (12, 256, 64), (2, 4096, 64),     # 16-byte path, whole tiles
    (3, 200, 72), (2, 72, 136),       # 16-byte path, partial t and d tiles
    (5, 64, 7), (5, 40, 7), (3, 130, 70)])   # element path
def test_transpose_hd_is_bit_exact(B, T, D):
    x = randn16((B, T, D), 18)
    y = G.empty((B, D, T), np.float16)
    dx = G.dev(x)
    G.call("hexlib_b200_transpose_hd_fp16", G.ptr(dx), G.ptr(y), B, T, D, G.stream())
    assert_bit_exact(G.host(y), np.ascontiguousarray(x.transpose(0, 2, 1)), "transpose_hd")


@pytest.mark.parametrize("S,p,m", [(256, 16, 2), (32, 4, 2), (48, 8, 3), (36, 6, 2)])
def test_patchify_is_bit_exact(S, p, m):
    img = rng(19).standard_normal((3, 2, S, S)).astype(np.float32)
    g = S // p
    attrs = {"patch": p, "temporal_patch": 2, "merge": m, "grid_h": g, "grid_w": g}
    want = ops.patchify((img,), attrs)[0]
    y = G.empty(want.shape, np.float32)
    di = G.dev(img)
    G.call("hexlib_b200_patchify_fp32", G.ptr(di), G.ptr(y), 3, 2, S, S, p, m, g, g, G.stream())
    assert_bit_exact(G.host(y), want, "patchify")


@pytest.mark.parametrize("S,p,m", [(512, 16, 2), (256, 16, 2), (64, 8, 2), (96, 4, 3)])
def test_patchify_to_fp16_is_patchify_then_cast_bit_for_bit(S, p, m):
    img = (rng(21).standard_normal((3, 2, S, S)) * 3).astype(np.float32)
    g = S // p
    attrs = {"patch": p, "temporal_patch": 2, "merge": m, "grid_h": g, "grid_w": g}
    want = ops.patchify((img,), attrs)[0].astype(np.float16)   # the cast op: nearest even
    y = G.empty(want.shape, np.float16)
    di = G.dev(img)
    G.call("hexlib_b200_patchify_fp16", G.ptr(di), G.ptr(y), 3, 2, S, S, p, m, g, g, G.stream())
    assert_bit_exact(G.host(y), want, "patchify -> fp16")


def test_patchify_matches_the_registrys_reshape_chain():
    # The oracle's scalar index map against the reference's own reshape /
    # transpose(2,5,3,6,0,1,4,7) formulation (structural.py:200-207).
    img = rng(20).standard_normal((3, 2, 32, 32)).astype(np.float32)
    x = img.reshape(3, 2, 8, 4, 8, 4).reshape(3, 2, 4, 2, 4, 4, 2, 4)
    chain = x.transpose(2, 5, 3, 6, 0, 1, 4, 7).reshape(64, 96)
    attrs = {"patch": 4, "temporal_patch": 2, "merge": 2, "grid_h": 8, "grid_w": 8}
    assert_bit_exact(ops.patchify((img,), attrs)[0], chain, "oracle patchify")


# ---- GEMMs -------------------------------------------------------------------------

ACT = {"none": 0, "gelu_tanh": 1, "gelu_erf": 2}


@pytest.mark.parametrize("M,K,N,act", [
    (256, 768, 768, "none"),
    (256, 768, 3072, "gelu_tanh"),
    (256, 3072, 768, "none"),
    (64, 3072, 3072, "gelu_erf"),
    (64, 3072, 1024, "none"),
    (256, 1536, 768, "none"),
    (200, 128, 200, "gelu_tanh"),   # M and N tails on the tensor-core path
    (1000, 64, 64, "none"),
    # N % 256 == 0 runs on CTA pairs (256-row tiles split over two SMs):
    (300, 768, 512, "none"),        # the second CTA's rows end inside its tile
    (128, 200, 256, "gelu_tanh"),   # the second CTA's rows are all past M; K tail
    (8192, 512, 2304, "none"),      # several tiles per pair, accumulators cycle
    (20, 40, 96, "gelu_erf"),       # K % 8 != 0 -> CUDA-core fallback
    (3, 64, 30, "none"),            # N % 8 != 0 -> fallback
])
def test_matmul_epilogue(M, K, N, act):
    a = randn16((M, K), 21, scale=1.0)
    w = randn16((K, N), 22, scale=0.02 if K >= 256 else 0.1)
    bias = (rng(23).standard_normal(N) * 0.02).astype(np.float32)
    y = G.empty((M, N), np.float16)
    da, dw, db = G.dev(a), G.dev(w), G.dev(bias)
    G.call("hexlib_b200_matmul_epilogue_fp16", G.ptr(da), G.ptr(dw), G.ptr(db), G.ptr(y),
           M, K, N, ACT[act], G.stream())
    assert_close_f16(G.host(y), oracle16("matmul_epilogue", (a, w, bias), {"act": act}),
                     what=f"matmul_epilogue {M}x{K}x{N} {act}")


def test_matmul_epilogue_gate_shape_unit_weights():
    # The benchmark's gate shape with N(0,1) weights: outputs ~ +-30, where one
    # fp16 step is 1/32 -- the bound is one rounding step.
    M, K, N = 256, 768, 768
    a, w = randn16((M, K), 24), randn16((K, N), 25)
    bias = rng(26).standard_normal(N).astype(np.float32)
    y = G.empty((M, N), np.float16)
    da, dw, db = G.dev(a), G.dev(w), G.dev(bias)
    G.call("hexlib_b200_matmul_epilogue_fp16", G.ptr(da), G.ptr(dw), G.ptr(db), G.ptr(y),
           M, K, N, 0, G.stream())
    assert_close_f16(G.host(y), oracle16("matmul_epilogue", (a, w, bias), {"act": "none"}),
                     what="gate shape, unit weights")


def test_matmul_epilogue_residual():
    M, K, N = 512, 768, 768
    a, w = randn16((M, K), 27), randn16((K, N), 28, scale=0.02)
    r = randn16((M, N), 29)
    bias = (rng(30).standard_normal(N) * 0.02).astype(np.float32)
    y = G.empty((M, N), np.float16)
    da, dw, db, dr = G.dev(a), G.dev(w), G.dev(bias), G.dev(r)
    G.call("hexlib_b200_matmul_epilogue_residual_fp16", G.ptr(da), G.ptr(dw), G.ptr(db),
           G.ptr(dr), G.ptr(y), M, K, N, 0, G.stream())
    from oracle import ops
    from oracle.executor import matmul_epilogue_residual_chain
    af, wf = a.astype(np.float32), w.astype(np.float32)
    want = matmul_epilogue_residual_chain(af, wf, bias, r.astype(np.float32))
    product = ops.store(ops.matmul_epilogue((af, wf, bias), {"act": "none"})[0], "fp16")
    assert_close_f16(G.host(y), want, what="matmul_epilogue + residual", inner=product)


@pytest.mark.parametrize("Bn,M,K,N", [
    (12, 256, 64, 256),    # QK^T at 256^2
    (12, 256, 256, 64),    # PV at 256^2
    (3, 40, 128, 200),     # the matmul harness shape
    (2, 1024, 64, 1024),   # QK^T at 512^2, two heads
    (4, 64, 16, 64),       # tiny head dim
    (3, 200, 64, 512),     # pair tiles with an M tail inside each batch entry
])
def test_matmul_batched(Bn, M, K, N):
    a = randn16((Bn, M, K), 31)
    b = randn16((Bn, K, N), 32, scale=1.0 / np.sqrt(K))
    y = G.empty((Bn, M, N), np.float16)
    da, db = G.dev(a), G.dev(b)
    G.call("hexlib_b200_matmul_fp16", G.ptr(da), G.ptr(db), G.ptr(y), Bn, M, K, N, G.stream())
    assert_close_f16(G.host(y), oracle16("matmul", (a, b), {}), what=f"matmul {Bn}x{M}x{K}x{N}")


def test_matmul_catches_a_transposed_operand():
    # The near-miss the reference harness plants: B read as [N, K].
    Bn, M, K, N = 2, 128, 64, 128
    a, b = randn16((Bn, M, K), 33), randn16((Bn, K, N), 34)
    y = G.empty((Bn, M, N), np.float16)
    da, db = G.dev(a), G.dev(b)
    G.call("hexlib_b200_matmul_fp16", G.ptr(da), G.ptr(db), G.ptr(y), Bn, M, K, N, G.stream())
    got = G.host(y).astype(np.float64)
    wrong = a.astype(np.float64) @ np.ascontiguousarray(b.transpose(0, 2, 1)).reshape(Bn, K, N)
    assert np.abs(got - wrong).max() > 1.0


def test_invalid_arguments_are_refused_not_run():
    assert G.call_rc("hexlib_b200_softmax_fp16", 0, 0, 4, 0, 0) == 6      # C = 0
    assert G.call_rc("hexlib_b200_rope_2d_fp16", 0, 0, 0, 0, 4, 2, 7, 0) == 6  # odd D
    assert G.call_rc("hexlib_b200_matmul_epilogue_fp16", 0, 0, 0, 0, 4, 8, 8, 3, 0) == 6
    assert G.call_rc("hexlib_b200_patchify_fp32", 1, 1, 3, 2, 30, 30, 16, 2, 2, 2, 0) == 6
