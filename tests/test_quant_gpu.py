"""q4_0 / q8_0 weights on the GPU: the dequantization kernels bit for bit,
matmul_epilogue with a quantized weight against the oracle and against the
reference's own scalar kernel (kernels/matmul_epilogue_fp16/baseline.c, when
oracle/_ref is built), the reference's own batch blob and arena image run
through the dispatcher, and a quantized encoder plan that gives exactly the
bits of the fp16 plan fed the dequantized weights."""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import quant, wholeplan, wire
from hexlib_b200.session import Session
from oracle import cref, executor
from oracle import quant as oq
from tests import gpu_util as U
from tests.tolerance import assert_bit_exact, assert_close_f16

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
Z = np.load(os.path.join(GOLDEN, "quant.npz"))
ACT = {"none": 0, "gelu_tanh": 1, "gelu_erf": 2}


def rng(seed):
    return np.random.default_rng(seed)


def _dev_bytes(raw: bytes):
    return U.dev(np.frombuffer(raw, np.uint8).copy())


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
@pytest.mark.parametrize("K,N", [(10, 96), (768, 2304), (3, 32)])
def test_dequantization_is_bit_exact(dtype, K, N):
    x = Z["x"] if (K, N) == (10, 96) else (rng(K + N).standard_normal((K, N)) * 0.05).astype(np.float32)
    raw = quant.quantize(x, dtype)
    y = U.empty((K, N), np.float16)
    dw = _dev_bytes(raw)                  # held until the kernel has run
    U.call(f"hexlib_b200_dequant_{dtype}_fp16", U.ptr(dw), U.ptr(y), K, N, U.stream())
    assert_bit_exact(U.host(y), oq.dequantize_f16(raw, (K, N), dtype), f"dequant {dtype}")


def _run_quant_gemm(dtype, a, raw, bias, M, K, N, act, ws_bytes=None):
    y = U.empty((M, N), np.float16)
    ws = U.empty((K * N,), np.float16)
    nb = K * N * 2 if ws_bytes is None else ws_bytes
    # device copies held in locals until the launches have completed
    da, dw, db = U.dev(a), _dev_bytes(raw), U.dev(bias)
    rc = U.call_rc(f"hexlib_b200_matmul_epilogue_{dtype}", U.ptr(da), U.ptr(dw), U.ptr(db),
                   U.ptr(y), M, K, N, ACT[act], U.ptr(ws), ctypes.c_uint64(nb), U.stream())
    U.host(y)
    return rc, y


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,K,N,act", [
    (256, 768, 768, "none"),
    (256, 768, 3072, "gelu_tanh"),
    (64, 3072, 1024, "gelu_erf"),
    (200, 128, 224, "none"),          # M and N tails; N a multiple of 32, not of 64
])
def test_matmul_epilogue_with_a_quantized_weight(dtype, M, K, N, act):
    a = (rng(1).standard_normal((M, K))).astype(np.float16)
    w = (rng(2).standard_normal((K, N)) * (0.02 if K >= 256 else 0.1)).astype(np.float32)
    bias = (rng(3).standard_normal(N) * 0.02).astype(np.float32)
    raw = quant.quantize(w, dtype)
    rc, y = _run_quant_gemm(dtype, a, raw, bias, M, K, N, act)
    assert rc == U.OK
    want = oq.matmul_epilogue_quant(a, raw, bias, K, N, dtype, act)
    assert_close_f16(U.host(y), want.astype(np.float16), what=f"{dtype} {M}x{K}x{N} {act}")


@pytest.mark.skipif(not cref.available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("act", ["none", "gelu_tanh"])
def test_q4_0_matmul_agrees_with_the_reference_scalar_kernel(act):
    M, K, N = 64, 768, 256
    a = (rng(4).standard_normal((M, K))).astype(np.float16)
    w = (rng(5).standard_normal((K, N)) * 0.02).astype(np.float32)
    bias = (rng(6).standard_normal(N) * 0.02).astype(np.float32)
    raw = np.frombuffer(quant.quantize_q4_0(w), np.uint8).copy()
    ref = np.zeros((M, N), np.float16)
    cref.call("matmul_epilogue_fp16", a, raw, bias, ref, M, K, N, ACT[act])
    rc, y = _run_quant_gemm("q4_0", a, raw.tobytes(), bias, M, K, N, act)
    assert rc == U.OK
    assert_close_f16(U.host(y), ref, what=f"vs baseline.c {act}")


def test_a_short_workspace_or_a_ragged_n_is_refused():
    M, K, N = 16, 64, 64
    a = np.zeros((M, K), np.float16)
    raw = quant.quantize_q4_0(np.zeros((K, N), np.float32))
    bias = np.zeros(N, np.float32)
    rc, _ = _run_quant_gemm("q4_0", a, raw, bias, M, K, N, "none", ws_bytes=K * N * 2 - 2)
    assert rc == 6                                    # ERR_INVAL_PARAMS
    rc = U.call_rc("hexlib_b200_dequant_q4_0_fp16", 0, 0, 4, 40, U.stream())
    assert rc == 6


def test_the_references_own_q4_0_batch_runs_through_the_dispatcher():
    """build_whole_plan_batch of the tiny encoder, by the reference, with the
    arena image it staged (q4_0 weights, the image) -- one buffer, one blob."""
    blob = Z["plan_blob"].tobytes()
    payload = Z["plan_payload"]
    hdr = wire.HDR.unpack_from(blob, 0)
    assert hdr[3] == 1
    _, size, fd, flags = wire.BUF.unpack_from(blob, hdr[6])
    assert size == payload.size and flags == 0
    off, nbytes = (int(v) for v in Z["plan_out"])
    want = Z["plan_expected"]
    with Session(0) as s:
        s.mmap(fd, size, 1)
        s.write(fd, 0, np.ascontiguousarray(payload))
        cap = wire.response_capacity(hdr[5])
        rsp = (ctypes.c_uint8 * cap)()
        rlen = ctypes.c_uint32()
        buf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        for _ in range(2):                       # capture, then replay
            rc = s._L.hexlib_b200_invoke(s._h, ctypes.addressof(buf), len(blob),
                                         ctypes.addressof(rsp), cap, ctypes.byref(rlen))
            r = wire.unpack_response(bytes(rsp[:rlen.value]))
            assert rc == 1 and r.ok and r.n_ops == hdr[5]
        got = np.empty(want.shape, np.float16)
        s.read(fd, off, got)
    assert nbytes == got.nbytes
    rel = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert rel < 1e-2, rel
    assert json.loads(Z["plan_quantized"].tobytes())[0] == "blk0.w_fc1"


@pytest.fixture(scope="module")
def enc256():
    return G.qwen35_at(256)


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
def test_a_quantized_plan_gives_the_bits_of_the_fp16_plan_on_dequantized_weights(enc256, dtype):
    cfg_q = G.qwen35_at(256, weight_dtype=dtype)
    gq = G.build_vision_encoder(cfg_q)
    wq = F.weights(cfg_q, 0, gq)
    g16 = G.build_vision_encoder(enc256)
    w16 = dict(wq)
    for n, t in gq.tensors.items():
        if t.const and t.dtype == dtype:
            w16[n] = oq.dequantize_f16(quant.quantize(wq[n], dtype), t.shape, dtype)
    imgs = F.images(enc256, 2, 3)
    outs = []
    for g, w in ((gq, wq), (g16, w16)):
        ep = G.compile_for_cuda(g, residual=True)
        plan = wholeplan.build_cuda_plan(ep, w, alias=True)
        with Session(0) as s:
            s.load(plan, max_images=2)
            outs.append(s.run(np.ascontiguousarray(imgs)))
    np.testing.assert_array_equal(outs[0], outs[1])
    ref = executor.run(G.compile_for_cuda(g16), dict(w16, image=imgs[0]))["merger.out"]
    rel = np.abs(outs[1][0].astype(np.float64) - ref).max() / np.abs(ref).max()
    assert rel < 1e-2, rel


def _dequantized_feeds(gq, wq, dtype):
    w16 = dict(wq)
    for n, t in gq.tensors.items():
        if t.const and t.dtype == dtype:
            w16[n] = oq.dequantize_f16(quant.quantize(wq[n], dtype), t.shape, dtype)
    return w16


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
def test_a_quantized_plan_with_every_default_rewrite_gives_the_fp16_plans_bits(enc256, dtype):
    """With the RoPE and residual epilogues and the packed q/k/v GEMM, the
    quantized plan's GEMMs read the session's fp16 copies of the weights: the
    same kernels, the same bits as the fp16 plan fed the dequantized weights."""
    cfg_q = G.qwen35_at(256, weight_dtype=dtype)
    gq = G.build_vision_encoder(cfg_q)
    wq = F.weights(cfg_q, 0, gq)
    g16 = G.build_vision_encoder(enc256)
    imgs = F.images(enc256, 2, 4)
    outs = []
    for g, w in ((gq, wq), (g16, _dequantized_feeds(gq, wq, dtype))):
        plan = wholeplan.build_cuda_plan(G.compile_for_cuda(g, **G.DEFAULT_REWRITES), w,
                                         alias=True)
        with Session(0) as s:
            s.load(plan, max_images=2)
            outs.append(s.run(np.ascontiguousarray(imgs)))
    assert "matmul_epilogue_rope" in plan.kinds
    np.testing.assert_array_equal(outs[0], outs[1])


def test_rewriting_a_quantized_weight_refreshes_the_sessions_copy(enc256):
    """The quantized bytes are the source of truth: new consts written into
    the mapped buffer are seen by the next replay of the cached graph."""
    cfg_q = G.qwen35_at(256, weight_dtype="q4_0")
    gq = G.build_vision_encoder(cfg_q)
    ep = G.compile_for_cuda(gq, **G.DEFAULT_REWRITES)
    p1 = wholeplan.build_cuda_plan(ep, F.weights(cfg_q, 0, gq), alias=True)
    p2 = wholeplan.build_cuda_plan(ep, F.weights(cfg_q, 5, gq), alias=True)
    assert p1.blob == p2.blob and p1.const_payload != p2.const_payload
    imgs = np.ascontiguousarray(F.images(enc256, 1, 6))
    with Session(0) as s:
        s.load(p1, max_images=1)
        out1 = s.run(imgs)
        s.write(wholeplan.CONST_FD, 0, np.frombuffer(p2.const_payload, np.uint8))
        out2 = s.run(imgs)                                         # cached graph replay
    with Session(0) as s:
        s.load(p2, max_images=1)
        want2 = s.run(imgs)
    assert not np.array_equal(out1, out2)
    np.testing.assert_array_equal(out2, want2)
