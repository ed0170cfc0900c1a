"""LayerNorm folded into the GEMM that consumes it: the row statistics
kernel against the oracle's float64 statistics, the folded GEMM (plain,
GELU and RoPE epilogues) against the oracle's layernorm -> matmul_epilogue
chain, and a whole encoder plan with every layernorm that feeds a GEMM folded
against the unfused oracle plan."""
from __future__ import annotations

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan
from hexlib_b200.session import Session
from oracle import executor, ops
from tests import gpu_util as U
from tests.tolerance import assert_close_f16

pytestmark = pytest.mark.gpu

ACT = {"none": 0, "gelu_tanh": 1, "gelu_erf": 2}


def rng(seed):
    return np.random.default_rng(seed)


def rows(R, C, seed, offset=0.0):
    # a per-row offset, so the folded epilogue's mean correction is exercised
    x = rng(seed).standard_normal((R, C)) + offset * rng(seed + 1).standard_normal((R, 1))
    return x.astype(np.float16)


def ln_params(C, seed):
    gamma = (1.0 + 0.1 * rng(seed).standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng(seed + 1).standard_normal(C)).astype(np.float32)
    return gamma, beta


@pytest.mark.parametrize("R,C", [(1024, 768), (300, 1024), (65, 768), (17, 200)])
def test_ln_stats_match_float64_statistics(R, C):
    x = rows(R, C, 1, offset=3.0)
    st = U.empty((R, 2), np.float32)
    dx = U.dev(x)
    U.call("hexlib_b200_ln_stats_fp16", U.ptr(dx), U.ptr(st), R, C, 1e-6, U.stream())
    got = U.host(st)
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1)
    rstd = 1.0 / np.sqrt(((xd - mean[:, None]) ** 2).mean(axis=1) + 1e-6)
    np.testing.assert_allclose(got[:, 0], mean, rtol=0, atol=1e-5 * (1 + np.abs(mean).max()))
    np.testing.assert_allclose(got[:, 1], rstd, rtol=2e-6)


def _stats(x, eps):
    R, C = x.shape
    st = U.empty((R, 2), np.float32)
    dx = U.dev(x)
    U.call("hexlib_b200_ln_stats_fp16", U.ptr(dx), U.ptr(st), R, C, eps, U.stream())
    U.host(st)
    return st


def _oracle_chain(x, gamma, beta, w, b, act, eps):
    (y,) = ops.layernorm((x, gamma, beta), {"eps": eps})          # fp16, as stored
    (out,) = ops.matmul_epilogue((y.astype(np.float32), w.astype(np.float32), b),
                                 {"act": act})
    return out


@pytest.mark.parametrize("M,K,N,act,offset", [
    (512, 768, 3072, "gelu_tanh", 0.0),
    (512, 768, 2304, "none", 2.0),
    (300, 768, 256, "gelu_erf", 0.5),       # M tail
    (128, 1024, 512, "none", 0.0),
])
def test_folded_gemm_matches_layernorm_then_matmul(M, K, N, act, offset):
    x = rows(M, K, 3, offset)
    gamma, beta = ln_params(K, 5)
    w = (rng(7).standard_normal((K, N)) * 0.03).astype(np.float16)
    b = (rng(8).standard_normal(N) * 0.02).astype(np.float32)
    eps = 1e-6
    wf = wholeplan.ln_fold_w(gamma, w)
    cols = wholeplan.ln_fold_cols(gamma, beta, w, b)
    st = _stats(x, eps)
    y = U.empty((M, N), np.float16)
    dx, dw, dc = U.dev(x), U.dev(wf), U.dev(cols)
    U.call("hexlib_b200_matmul_epilogue_ln_fp16", U.ptr(dx), U.ptr(dw), U.ptr(dc), U.ptr(st),
           U.ptr(y), M, K, N, ACT[act], U.stream())
    want = _oracle_chain(x, gamma, beta, w, b, act, eps)
    # the unfused chain rounds layernorm(x) to fp16, the folded GEMM rounds
    # diag(gamma) W instead: two fp16 roundings of the same size, then one
    # rounding of the result each -- within two steps of each other
    assert_close_f16(U.host(y), want.astype(np.float16), what=f"{M}x{K}x{N} {act}", ulps=2)


@pytest.mark.parametrize("T,H,n_img", [(256, 12, 2), (1024, 12, 1)])
def test_folded_rope_gemm_matches_the_unfused_chain(T, H, n_img):
    D, K = 64, H * 64
    N = 3 * H * D
    M = T * n_img
    x = rows(M, K, 11, offset=1.0)
    gamma, beta = ln_params(K, 13)
    w = (rng(15).standard_normal((K, N)) * 0.03).astype(np.float16)
    b = (rng(16).standard_normal(N) * 0.02).astype(np.float32)
    side = int(round(T ** 0.5))
    r, c = np.divmod(np.arange(T), side)
    f = rng(17).uniform(-3, 3, (T, 32)).astype(np.float32)
    ang = np.concatenate([f[r, :16], f[c, 16:]], 1)
    ang = np.concatenate([ang, ang], 1)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    seg_cos, seg_sin, seg_idx = wholeplan.rope_segments(cos, sin)
    n_seg = int(seg_idx.max()) + 1
    segtab = np.ascontiguousarray(np.stack([seg_cos, seg_sin], axis=1)[:n_seg])
    eps = 1e-6
    st = _stats(x, eps)
    wf = wholeplan.ln_fold_w(gamma, w)
    cols = wholeplan.ln_fold_cols(gamma, beta, w, b)
    got = U.empty((M, N), np.float16)
    dx, dw, dc, dt, di = U.dev(x), U.dev(wf), U.dev(cols), U.dev(segtab), U.dev(seg_idx)
    U.call("hexlib_b200_matmul_epilogue_ln_rope_fp16", U.ptr(dx), U.ptr(dw), U.ptr(dc),
           U.ptr(st), U.ptr(dt), U.ptr(di), n_seg, U.ptr(got), M, K, N, 0, 2 * H * D, T,
           U.stream())
    # the oracle chain: layernorm stored as fp16, the three projections
    # stored as fp16, rope_2d of q and k stored as fp16
    (y,) = ops.layernorm((x, gamma, beta), {"eps": eps})
    (proj,) = ops.matmul_epilogue((y.astype(np.float32), w.astype(np.float32), b),
                                  {"act": "none"})
    proj = ops.store(proj, "fp16").reshape(n_img, T, 3, H, D)
    want = proj.astype(np.float64).copy()
    for n in range(n_img):
        for sec in range(2):
            (rot,) = ops.rope_2d((proj[n, :, sec].astype(np.float32), cos, sin), {})
            want[n, :, sec] = ops.store(rot, "fp16")
    # Two paths that round differently ahead of the GEMM (layernorm(x) vs
    # diag(gamma) W), each within 2e-3 of the exact value; the rotation adds
    # two such errors: 4e-3 apart at most, or three fp16 steps where wider.
    assert_close_f16(U.host(got).reshape(want.shape), want, atol=4e-3, ulps=3,
                     what=f"T={T}")


def test_folded_gemm_refuses_what_it_cannot_serve():
    # N not a multiple of 256; null statistics
    assert U.call_rc("hexlib_b200_matmul_epilogue_ln_fp16", 0, 0, 0, 0, 0, 16, 64, 128, 0,
                     U.stream()) == 6
    x = U.empty((16, 64), np.float16)
    assert U.call_rc("hexlib_b200_matmul_epilogue_ln_fp16", U.ptr(x), U.ptr(x), U.ptr(x), 0,
                     U.ptr(x), 16, 64, 256, 0, U.stream()) == 6


@pytest.mark.parametrize("size", [256, 512])
def test_encoder_with_folded_layernorms_matches_the_oracle(size):
    cfg = G.qwen35_at(size)
    g = G.build_vision_encoder(cfg)
    w = F.weights(cfg, 0, g)
    imgs = F.images(cfg, 2, 23)
    ep = G.compile_for_cuda(g, residual=True, qkv=True, rope_epilogue=True, ln_fold=True)
    plan = wholeplan.build_cuda_plan(ep, w, alias=True)
    assert plan.kinds.count("ln_stats") == 24
    assert plan.kinds.count("matmul_epilogue_ln_rope") == 12
    assert plan.kinds.count("matmul_epilogue_ln") == 12
    with Session(0) as s:
        s.load(plan, max_images=2)
        out = s.run(np.ascontiguousarray(imgs))
    for i in range(2):
        ref = executor.run(G.compile_for_cuda(g), dict(w, image=imgs[i]))["merger.out"]
        err = np.abs(out[i].astype(np.float64) - ref).max() / np.abs(ref).max()
        assert err < 1e-2, f"image {i}: relative error {err:.3e}"
