"""Plans loaded from the reference's own `Compiled` JSON artefacts
(hexlib/graph/compiled.py:90-168, written by tests/golden/make_golden.py from
the reference) run through the CUDA batch path and match the oracle: the
tiny fp16 plan against the reference interpreter's own output, and the 256^2
fp16-weight plan -- as loaded, and with the CUDA-only rewrites applied to it
-- against the oracle's replay of the same plan."""
from __future__ import annotations

import gzip
import os

import numpy as np
import pytest

from hexlib_b200 import feeds as F
from hexlib_b200 import graph as G
from hexlib_b200 import wholeplan
from hexlib_b200.session import Session
from oracle import executor

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def run(ep, feeds, imgs):
    plan = wholeplan.build_cuda_plan(ep, feeds, alias=True)
    with Session(0) as s:
        s.load(plan, max_images=len(imgs))
        return s.run(np.ascontiguousarray(imgs)), plan


def test_the_tiny_json_plan_matches_the_reference_interpreter():
    ep = G.from_compiled_json(open(os.path.join(GOLDEN, "tiny_compiled.json")).read())
    z = np.load(os.path.join(GOLDEN, "tiny.npz"))
    feeds = {k[6:]: z[k] for k in z.files if k.startswith("feed::")}
    for n, t in ep.graph.tensors.items():
        if n in feeds and t.dtype == "fp16":
            feeds[n] = np.asarray(feeds[n], np.float16)
    img = feeds.pop("image")
    out, plan = run(ep, feeds, img[None])
    assert rel_err(out[0], z["interp_fp16_fp16"]) < 1e-2
    assert rel_err(out[0], executor.run(ep, dict(feeds, image=img))[plan.outputs[0]]) < 1e-2


@pytest.fixture(scope="module")
def json256():
    with gzip.open(os.path.join(GOLDEN, "qwen35_256_compiled.json.gz"), "rt") as fh:
        ep = G.from_compiled_json(fh.read())
    cfg = G.qwen35_at(256)
    w = F.weights(cfg, 0, G.build_vision_encoder(cfg))
    imgs = F.images(cfg, 2, 5)
    refs = [executor.run(ep, dict(w, image=imgs[i]))["merger.out"] for i in range(2)]
    return ep, w, imgs, refs


def test_the_256_json_plan_matches_the_oracle(json256):
    ep, w, imgs, refs = json256
    out, plan = run(ep, w, imgs)
    # the blob carries every step but the reshapes, which alias their input
    assert plan.n_ops == sum(1 for st in ep.plan.steps if st.op.kind != "reshape")
    for i in range(2):
        assert rel_err(out[i], refs[i]) < 1e-2, f"image {i}"


def test_the_256_json_plan_with_the_cuda_rewrites_matches_the_oracle(json256):
    ep, w, imgs, refs = json256
    rw = G.rewrite_compiled(ep, **G.DEFAULT_REWRITES)
    out, plan = run(rw, w, imgs)
    assert "attention_qkv" in plan.kinds and "matmul_epilogue_rope" in plan.kinds
    for i in range(2):
        assert rel_err(out[i], refs[i]) < 1e-2, f"image {i}"
