"""The packed q/k/v path: one GEMM over [wq|wk|wv] with RoPE in its epilogue,
attention straight from the packed [T, 3, H, D] tensor into [T, H, D]."""
from __future__ import annotations

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan
from hexlib_b200.session import Session
from oracle import executor, ops
from tests import gpu_util as U
from tests.tolerance import assert_close_f16, f16_ulp

pytestmark = pytest.mark.gpu


def r16(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float16)


@pytest.mark.parametrize("T,H,n_img,grid", [(256, 12, 2, False), (64, 4, 3, False),
                                             (1024, 12, 1, False), (1024, 12, 4, True),
                                             (256, 16, 3, True)])
def test_rope_gemm_equals_three_projections_then_rope(T, H, n_img, grid):
    D, K = 64, H * 64
    M = T * n_img
    a = r16((M, K), 1)
    ws = [r16((K, H * D), 2 + i, 0.05) for i in range(3)]
    bs = [(np.random.default_rng(5 + i).standard_normal(H * D) * 0.02).astype(np.float32)
          for i in range(3)]
    ang = np.random.default_rng(9).uniform(-3, 3, (T, D // 2)).astype(np.float32)
    w = np.concatenate(ws, 1)
    b = np.concatenate(bs)
    if grid:
        # a 2-D table: dims [0,16) follow the patch row, [16,32) its column
        side = int(round(T ** 0.5))
        r, c = np.divmod(np.arange(T), side)
        ang = np.concatenate([ang[r, :16], ang[c, 16:]], 1)
    ang = np.concatenate([ang, ang], 1)       # rotate-half tables: dims i, i + 32 equal
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    seg_cos, seg_sin, seg_idx = wholeplan.rope_segments(cos, sin)
    n_seg = int(seg_idx.max()) + 1
    y = U.empty((M, 3 * H * D), np.float16)
    da, dw, db = U.dev(a), U.dev(w), U.dev(b)
    dc, ds, dx = U.dev(seg_cos[:n_seg]), U.dev(seg_sin[:n_seg]), U.dev(seg_idx)
    U.call("hexlib_b200_matmul_epilogue_rope_fp16", U.ptr(da), U.ptr(dw), U.ptr(db), U.ptr(dc),
           U.ptr(ds), U.ptr(dx), n_seg, U.ptr(y), M, K, 3 * H * D, 0, 2 * H * D, T, U.stream())
    got = U.host(y).reshape(n_img, T, 3, H, D)
    af = a.astype(np.float32)
    for i, which in enumerate("qkv"):
        proj = ops.store(ops.matmul_epilogue((af, ws[i].astype(np.float32), bs[i]),
                                             {"act": "none"})[0], "fp16")
        proj = proj.reshape(n_img, T, H, D)
        for n in range(n_img):
            if which == "v":
                assert_close_f16(got[n, :, i], proj[n], what=f"v image {n}")
                continue
            want = ops.store(ops.rope_2d((proj[n], cos, sin), {})[0], "fp16")
            # y = x*cos -/+ partner*sin: each of the two GEMM outputs may sit one
            # fp16 step from the oracle's fp32 summation order, and y is rounded
            # once more -- the bound is those steps, weighted as the rotation does.
            partner = np.concatenate([proj[n][..., D // 2:], proj[n][..., :D // 2]], -1)
            bound = (f16_ulp(proj[n]) * np.abs(cos)[:, None, :]
                     + f16_ulp(partner) * np.abs(sin)[:, None, :] + f16_ulp(want))
            err = np.abs(got[n, :, i].astype(np.float64) - want)
            assert np.all(err <= np.maximum(2e-3, bound)), \
                f"{which} image {n}: worst excess {np.max(err - np.maximum(2e-3, bound)):.3e}"
            assert np.mean(err == 0) > 0.99


@pytest.mark.parametrize("inplace", [True, False])
@pytest.mark.parametrize("T,H,n_img", [(256, 12, 2), (64, 4, 1)])
def test_rope_qk_rotates_q_and_k_sections_only(T, H, n_img, inplace):
    D = 64
    qkv = r16((n_img, T, 3, H, D), 31)
    ang = np.random.default_rng(33).uniform(-3, 3, (T, D)).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    d, dc, ds = U.dev(qkv), U.dev(cos), U.dev(sin)
    out = d if inplace else U.empty(qkv.shape, np.float16)
    U.call("hexlib_b200_rope_qk_fp16", U.ptr(d), U.ptr(dc), U.ptr(ds), U.ptr(out),
           n_img * T, H, D, T, U.stream())
    got = U.host(out)
    for n in range(n_img):
        for sec in range(2):
            want = ops.store(ops.rope_2d((qkv[n, :, sec].astype(np.float32), cos, sin), {})[0],
                             "fp16").astype(np.float16)
            np.testing.assert_array_equal(got[n, :, sec], want)
        np.testing.assert_array_equal(got[n, :, 2], qkv[n, :, 2])


def exact(q, k, v, scale):
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = np.einsum("thd,shd->hts", q, k) * scale
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hts,shd->thd", p, v).astype(np.float16).astype(np.float64)


@pytest.mark.parametrize("B,T,H", [(2, 256, 12), (1, 1024, 12), (3, 200, 4), (2, 64, 2)])
def test_attention_over_the_packed_projection(B, T, H):
    qkv = r16((B, T, 3, H, 64), 11 + T)
    ctx = U.empty((B, T, H, 64), np.float16)
    d = U.dev(qkv)
    U.call("hexlib_b200_attention_qkv_fp16", U.ptr(d), U.ptr(ctx), B, T, H, 64, 0.125, U.stream())
    got = U.host(ctx)
    for b in range(B):
        want = exact(qkv[b, :, 0], qkv[b, :, 1], qkv[b, :, 2], 0.125)
        assert_close_f16(got[b], want, what=f"image {b}")


def test_packed_attention_refuses_what_it_cannot_serve():
    assert U.call_rc("hexlib_b200_attention_qkv_fp16", 0, 0, 1, 64, 2, 32, 0.125, 0) == 6
    assert U.call_rc("hexlib_b200_attention_qkv_fp16", 0, 0, 1, 64, 2, 64, -1.0, 0) == 6


@pytest.mark.parametrize("rope_epilogue,patch_cast", [(False, False), (True, True)])
def test_fully_fused_encoder_matches_the_oracle(rope_epilogue, patch_cast):
    cfg = G.qwen35_at(256)
    g = G.build_vision_encoder(cfg)
    w = F.weights(cfg, 0, g)
    imgs = F.images(cfg, 2, 21)
    ep = G.compile_for_cuda(g, residual=True, qkv=True, rope_epilogue=rope_epilogue,
                            patch_cast=patch_cast)
    plan = wholeplan.build_cuda_plan(ep, w, alias=True)
    assert plan.kinds.count("attention_qkv") == 12
    assert plan.kinds.count("matmul_epilogue_rope") == (12 if rope_epilogue else 0)
    assert plan.kinds.count("patchify_cast") == (1 if patch_cast else 0)
    with Session(0) as s:
        s.load(plan, max_images=2)
        out = s.run(np.ascontiguousarray(imgs))
    for i in range(2):
        ref = executor.run(G.compile_for_cuda(g), dict(w, image=imgs[i]))["merger.out"]
        err = np.abs(out[i].astype(np.float64) - ref).max() / np.abs(ref).max()
        assert err < 1e-2, f"image {i}: relative error {err:.3e}"
