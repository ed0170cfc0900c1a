"""The plan bench.py measures, at the sizes it measures, against the oracle.

bench.py's workload is the 512^2 encoder with every default CUDA-path rewrite
(graph.DEFAULT_REWRITES: fused attention over the packed q/k/v projection,
RoPE in the qkv GEMM's epilogue, residual epilogues, patchify writing fp16
rows) on an aliased arena. Here that plan runs on 8 images -- M = 8192 rows
per GEMM, so the persistent GEMMs cycle tiles through both TMEM accumulators
and the residual GEMMs prefetch the next tile's residual -- and at 1024^2 on
one image; every image's embeddings must be within 1e-2 relative (max |diff|
/ max |ref|) of the oracle's replay of the unfused plan on the same feeds.

The oracle replays run in a `spawn` process pool started before this module's
first GPU call, concurrently with the GPU work.
"""
from __future__ import annotations

import multiprocessing as mp
import os

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan
from hexlib_b200.session import Session

pytestmark = pytest.mark.gpu

N512 = 8


def _oracle_embeddings(job):
    """One image through the oracle (runs in a spawned worker)."""
    size, seed, index, threads = job
    import threadpoolctl

    from hexlib_b200 import feeds as Fw
    from hexlib_b200 import graph as Gw
    from oracle import executor
    with threadpoolctl.threadpool_limits(threads):
        cfg = Gw.qwen35_at(size)
        g = Gw.build_vision_encoder(cfg)
        w = Fw.weights(cfg, 0, g)
        img = Fw.images(cfg, index + 1, seed)[index]
        return executor.run(Gw.compile_for_cuda(g), dict(w, image=img))["merger.out"]


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.fixture(scope="module")
def oracle_results():
    """Oracle embeddings for the 512^2 images and the 1024^2 image, computed
    in the background while the GPU tests below run."""
    cores = os.cpu_count() or 4
    workers = max(1, min(N512 + 1, cores // 2))
    threads = max(1, cores // workers)
    jobs = [(512, 1, i, threads) for i in range(N512)] + [(1024, 2, 0, threads)]
    pool = mp.get_context("spawn").Pool(workers)
    pending = [pool.apply_async(_oracle_embeddings, (j,)) for j in jobs]
    try:
        yield {(j[0], j[2]): p for j, p in zip(jobs, pending)}
    finally:
        pool.terminate()
        pool.join()


def _run_default_plan(size: int, seed: int, n: int):
    cfg = G.qwen35_at(size)
    g = G.build_vision_encoder(cfg)
    ep = G.compile_for_cuda(g, **G.DEFAULT_REWRITES)
    plan = wholeplan.build_cuda_plan(ep, F.weights(cfg, 0, g), alias=True)
    imgs = F.images(cfg, n, seed)
    with Session(0) as s:
        s.load(plan, max_images=n)
        out = s.run(np.ascontiguousarray(imgs))
    return plan, out


def test_the_bench_plan_at_512_on_8_images_matches_the_oracle(oracle_results):
    plan, out = _run_default_plan(512, 1, N512)
    kinds = set(plan.kinds)
    assert {"attention_qkv", "matmul_epilogue_rope", "matmul_epilogue_residual",
            "patchify_cast"} <= kinds
    assert out.shape == (N512, 256, 1024)
    errs = []
    for i in range(N512):
        ref = oracle_results[(512, i)].get(timeout=1200)
        errs.append(rel_err(out[i], ref))
    assert max(errs) < 1e-2, f"relative errors per image: {errs}"


def test_the_bench_plan_at_1024_on_one_image_matches_the_oracle(oracle_results):
    plan, out = _run_default_plan(1024, 2, 1)
    assert out.shape == (1, 1024, 1024)
    ref = oracle_results[(1024, 0)].get(timeout=1800)
    err = rel_err(out[0], ref)
    assert err < 1e-2, f"relative error {err:.3e}"
