"""The persistent kernels walk their tiles, items and rows in ascending or
descending order, alternating from one launch to the next on a host thread,
so that a consumer starts on the rows its producer wrote last. The order is a
schedule only: two consecutive calls of the same entry point -- one in each
order -- must give bit-identical outputs, on shapes with partial tiles and
more tiles than the device holds at once."""
from __future__ import annotations

import numpy as np
import pytest

from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def r16(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float16)


def twice(fn):
    """Outputs of two consecutive launches (opposite walk orders)."""
    a, b = fn(), fn()
    return U.host(a), U.host(b)


@pytest.mark.parametrize("M,K,N,act", [
    (40000, 768, 768, 0),      # pair tiles, many rounds, partial last row tile
    (9000, 768, 3072, 1),      # GELU, single-CTA 128 x 256 tiles where chosen
    (300, 256, 512, 0),
])
def test_gemm_is_the_same_in_either_order(M, K, N, act):
    a, w = r16((M, K), 1), r16((K, N), 2, 0.03)
    bias = (np.random.default_rng(3).standard_normal(N) * 0.02).astype(np.float32)
    da, dw, db = U.dev(a), U.dev(w), U.dev(bias)

    def run():
        y = U.empty((M, N), np.float16)
        U.call("hexlib_b200_matmul_epilogue_fp16", U.ptr(da), U.ptr(dw), U.ptr(db), U.ptr(y),
               M, K, N, act, U.stream())
        return y
    y0, y1 = twice(run)
    assert np.array_equal(y0.view(np.uint16), y1.view(np.uint16))


@pytest.mark.parametrize("M,K,N", [
    (20000, 768, 768),      # partial last pair tile
    (65536, 768, 768),      # the o-projection of the 512^2 x 64 encoder: 768 pair tiles,
                            # both TMEM accumulators cycling, next-tile residual prefetch (K <= 1024)
    (65536, 3072, 768),     # its fc2: K > 1024, no prefetch
])
def test_residual_gemm_matches_the_oracle_in_either_order(M, K, N):
    """At the encoder's own row counts each CTA pair runs many tiles; both
    orders must equal each other bit for bit and the unfused oracle chain
    (matmul_epilogue rounded to fp16, then the residual add) within the bar."""
    from oracle import executor
    from tests.tolerance import assert_close_f16
    a, w, r = r16((M, K), 4), r16((K, N), 5, 0.03), r16((M, N), 6)
    bias = (np.random.default_rng(7).standard_normal(N) * 0.02).astype(np.float32)
    da, dw, db, dr = U.dev(a), U.dev(w), U.dev(bias), U.dev(r)

    def run():
        y = U.empty((M, N), np.float16)
        U.call("hexlib_b200_matmul_epilogue_residual_fp16", U.ptr(da), U.ptr(dw), U.ptr(db),
               U.ptr(dr), U.ptr(y), M, K, N, 0, U.stream())
        return y
    y0, y1 = twice(run)
    from oracle import ops
    af, wf = a.astype(np.float32), w.astype(np.float32)
    ref = executor.matmul_epilogue_residual_chain(af, wf, bias, r.astype(np.float32))
    product = ops.store(ops.matmul_epilogue((af, wf, bias), {"act": "none"})[0], "fp16")
    assert_close_f16(y0, ref, what=f"residual GEMM {M}x{K}x{N}", inner=product)
    assert np.array_equal(y0.view(np.uint16), y1.view(np.uint16))


@pytest.mark.parametrize("B,T,H", [(12, 1024, 12), (3, 200, 4)])
def test_attention_is_the_same_in_either_order(B, T, H):
    qkv = r16((B, T, 3, H, 64), 8)
    d = U.dev(qkv)

    def run():
        ctx = U.empty((B, T, H, 64), np.float16)
        U.call("hexlib_b200_attention_qkv_fp16", U.ptr(d), U.ptr(ctx), B, T, H, 64, 0.125,
               U.stream())
        return ctx
    c0, c1 = twice(run)
    assert np.array_equal(c0.view(np.uint16), c1.view(np.uint16))


@pytest.mark.parametrize("R,C", [(70001, 768), (333, 1024), (65, 4096), (1000, 64)])
def test_layernorm_is_the_same_in_either_order(R, C):
    x = r16((R, C), 9)
    g = (1 + 0.1 * np.random.default_rng(10).standard_normal(C)).astype(np.float32)
    b = (0.1 * np.random.default_rng(11).standard_normal(C)).astype(np.float32)
    dx, dg, db = U.dev(x), U.dev(g), U.dev(b)

    def run():
        y = U.empty((R, C), np.float16)
        U.call("hexlib_b200_layernorm_fp16", U.ptr(dx), U.ptr(dg), U.ptr(db), U.ptr(y), R, C,
               1e-6, U.stream())
        return y
    y0, y1 = twice(run)
    assert np.array_equal(y0.view(np.uint16), y1.view(np.uint16))
