"""The batch path end to end on the GPU: one blob per plan, one CUDA graph per
(blob, image count), checked against the oracle's plan replay.

Final embeddings must be within 1e-2 relative (max |diff| / max |ref|) of
the oracle; everything the dispatcher promises about the response (statuses,
stop-at-first-failure, timings) is checked on real launches.
"""
from __future__ import annotations

import dataclasses
import os
import struct

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan, wire
from hexlib_b200.session import MODE_EAGER, B200Error, Session
from oracle import executor

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY16 = G.VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                     patch_size=4, temporal_patch_size=2, in_channels=3,
                     spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                     rope_theta=10000.0, image_size=32, act_dtype="fp16",
                     weight_dtype="fp16")


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def tiny_feeds():
    z = np.load(os.path.join(GOLDEN, "tiny.npz"))
    f = {k[6:]: z[k] for k in z.files if k.startswith("feed::")}
    g = G.build_vision_encoder(TINY16)
    for k, v in list(f.items()):
        if k in g.tensors and g.tensors[k].dtype == "fp16":
            f[k] = np.asarray(v, np.float16)
    return f, z


def run_plan(ep, wfeeds, imgs, alias=False, mode=0):
    plan = wholeplan.build_cuda_plan(ep, wfeeds, alias=alias)
    with Session(0) as s:
        s.load(plan, max_images=len(imgs))
        s.write_input(plan.inputs[0], np.ascontiguousarray(imgs), len(imgs))
        rsp = s.invoke(len(imgs), mode=mode)
        out = s.read_output(plan.outputs[0], len(imgs))
    return out, rsp, plan


def test_tiny_plan_matches_the_oracle_and_the_reference_interpreter():
    f, z = tiny_feeds()
    img = f.pop("image")
    ep = G.compile_for_cuda(G.build_vision_encoder(TINY16))
    out, rsp, plan = run_plan(ep, f, img[None])
    ref = executor.run(ep, dict(f, image=img))[plan.outputs[0]]
    assert rel_err(out[0], ref) < 1e-2
    assert rel_err(out[0], z["interp_fp16_fp16"]) < 1e-2
    assert rsp.ok and rsp.n_ops == plan.n_ops and rsp.arch == 100


@pytest.fixture(scope="module")
def enc256():
    cfg = G.qwen35_at(256)
    g = G.build_vision_encoder(cfg)
    w = F.weights(cfg, 0, g)
    imgs = F.images(cfg, 3, 7)
    refs = [executor.run(G.compile_for_cuda(g), dict(w, image=imgs[i]))["merger.out"]
            for i in range(2)]
    return cfg, g, w, imgs, refs


def test_encoder_256_unfused_plan_matches_the_oracle(enc256):
    cfg, g, w, imgs, refs = enc256
    out, rsp, plan = run_plan(G.compile_for_cuda(g), w, imgs[:2])
    assert plan.n_ops == 259
    for i in range(2):
        assert rel_err(out[i], refs[i]) < 1e-2, f"image {i}"


def test_batching_does_not_change_any_bit(enc256):
    cfg, g, w, imgs, refs = enc256
    ep = G.compile_for_cuda(g)
    many, _, _ = run_plan(ep, w, imgs)
    for i in range(3):
        one, _, _ = run_plan(ep, w, imgs[i:i + 1])
        np.testing.assert_array_equal(many[i], one[0])


def test_aliased_arena_gives_the_same_bits(enc256):
    cfg, g, w, imgs, refs = enc256
    ep = G.compile_for_cuda(g)
    a, _, pa = run_plan(ep, w, imgs[:2], alias=False)
    b, _, pb = run_plan(ep, w, imgs[:2], alias=True)
    assert pb.image_bytes < pa.image_bytes / 4
    np.testing.assert_array_equal(a, b)


def test_residual_fusion_matches_the_oracle(enc256):
    cfg, g, w, imgs, refs = enc256
    out, _, plan = run_plan(G.compile_for_cuda(g, residual=True), w, imgs[:2], alias=True)
    assert plan.kinds.count("matmul_epilogue_residual") == 24
    for i in range(2):
        assert rel_err(out[i], refs[i]) < 1e-2


def test_graph_replay_and_eager_mode_agree_bit_for_bit(enc256):
    cfg, g, w, imgs, refs = enc256
    plan = wholeplan.build_cuda_plan(G.compile_for_cuda(g), w, alias=True)
    with Session(0) as s:
        s.load(plan, max_images=2)
        s.write_input("image", np.ascontiguousarray(imgs[:2]), 2)
        r1 = s.invoke(2)
        o1 = s.read_output("merger.out", 2)
        r2 = s.invoke(2)                       # replay of the cached graph
        o2 = s.read_output("merger.out", 2)
        r3 = s.invoke(2, mode=MODE_EAGER)      # op by op, timed
        o3 = s.read_output("merger.out", 2)
    np.testing.assert_array_equal(o1, o2)
    np.testing.assert_array_equal(o1, o3)
    assert r1.ok and r2.ok and r3.ok
    assert r2.cycles_total > 0
    assert all(r.cycles > 0 for r in r3.results)
    assert [r.kind for r in r3.results] == [r.kind for r in r1.results]


def test_pipelined_batches_equal_one_at_a_time_runs(enc256):
    """Five different batches through a depth-2 pipeline (uploads and read-
    backs overlapping the other session's replay, page-locked host arrays)
    give each batch the bits a plain Session.run gives it."""
    import torch
    from hexlib_b200.session import Pipeline
    cfg, g, w, imgs, refs = enc256
    plan = wholeplan.build_cuda_plan(G.compile_for_cuda(g, residual=True), w, alias=True)
    batches = [np.ascontiguousarray(np.roll(imgs[:2], k, axis=-1)) for k in range(5)]
    shape = (2,) + tuple(plan.placements[plan.outputs[0]].shape)
    pin_in = [torch.from_numpy(b).pin_memory() for b in batches]
    pin_out = [torch.empty(shape, dtype=torch.float16).pin_memory() for _ in batches]
    with Session(0) as s:
        s.load(plan, max_images=2)
        want = [s.run(b) for b in batches]
        pipe = Pipeline(plan, max_images=2, sessions=[s])
        try:
            for b, o in zip(pin_in, pin_out):
                pipe.submit(b, o)
            pipe.drain()
        finally:
            pipe.close()
    for k in range(5):
        np.testing.assert_array_equal(pin_out[k].numpy(), want[k], err_msg=f"batch {k}")


def _patch_op_kind(blob: bytes, i: int, kind: int) -> bytes:
    b = bytearray(blob)
    off = wire.HDR.unpack_from(blob)[8] + i * wire.OP_SIZE
    struct.pack_into("<I", b, off, kind)
    return bytes(b)


def test_first_failing_op_stops_the_batch_after_running_the_ops_before_it():
    f, _ = tiny_feeds()
    img = f.pop("image")
    plan = wholeplan.build_cuda_plan(G.compile_for_cuda(G.build_vision_encoder(TINY16)), f)
    bad = _patch_op_kind(plan.blob, 3, 99)
    with Session(0) as s:
        s.load(plan, max_images=1)
        s.write_input("image", np.ascontiguousarray(img[None]), 1)
        plan.blob = bad
        s._blob = (type(s._blob)).from_buffer_copy(bad)
        with pytest.raises(B200Error) as e:
            s.invoke(1)
        rsp = e.value.response
        assert rsp.status == wire.STATUS["ERR_NO_KERNEL"] and rsp.n_ops == 4
        assert all(r.ok for r in rsp.results[:3]) and rsp.results[3].kind == 99
        # the ops before the failure really ran: the patch-embed output is set
        pe = s.read_output("patch_embed.out", 1)
        assert np.abs(pe).max() > 0


def test_unmapped_and_oversized_invocations_are_refused():
    f, _ = tiny_feeds()
    f.pop("image")
    plan = wholeplan.build_cuda_plan(G.compile_for_cuda(G.build_vision_encoder(TINY16)), f)
    with Session(0) as s:
        s.load(plan, max_images=2)
        with pytest.raises(ValueError):
            s.invoke(3)                               # more images than replicas
        s.munmap(wholeplan.IMAGE_FD)
        with pytest.raises(B200Error) as e:
            s.invoke(1)
        assert e.value.status == wire.STATUS["ERR_UNMAPPED"]
        info = s.hwinfo()
        assert info.arch == 100 and info.sm_count >= 100
