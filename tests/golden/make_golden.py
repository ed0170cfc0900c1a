"""Generate the golden fixtures in tests/golden/ FROM THE REFERENCE ITSELF.

Run where the reference's Python package (sriharshapy/hexlib) is importable:

    python tests/golden/make_golden.py /path/to/hexlib-checkout

It imports `hexlib` from that checkout and writes, with nothing of this
repository's code in the loop:

  tiny.npz      the reference's transformers golden (qwen35_vision_tiny.npz)
                mapped to graph feeds by hexlib's own loader, plus the
                reference interpreter's outputs for the fp32/fp32 and
                fp16/fp16 plans of that tiny encoder (fp16-declared consts
                are rounded to fp16 first, so every executor sees the same
                weights).
  ops.npz       seeded inputs and the op registry's own reference outputs for
                every op kind, at small shapes and at edge shapes.
  plans.json    the post-fusion graphs and plan orders `compile_model`
                produces for the tiny config and the 256/512/1024 encoders
                with fp16 weights.
  tiny_compiled.json   hexlib.graph.compiled.to_json of the tiny fp16 plan.
  wire.npz      blobs from hexlib.runtime.wire.pack_batch: a one-op batch and
                build_whole_plan_batch of the tiny fp16 plan, and response
                bytes for unpack_response.
  tables.npz    loader.rope_tables for the tiny and 256 configs.
  quant.npz     hexlib.exec.quant's q4_0 and q8_0 bytes and dequantized values
                for seeded blocks and the edge blocks its tests construct
                (exact halves, positive extremes, zero blocks, the q8_0 wrap
                case); and build_whole_plan_batch of the tiny fp16 plan --
                whose matmul_epilogue weights the builder quantizes to q4_0 --
                with its staged arena payload, the output's placement, and the
                reference interpreter's output when every quantized weight is
                replaced by its dequantized value rounded to fp16 (the
                arithmetic the DSP kernel performs, baseline.c:36-47).

  tiny_params.npz  the tiny golden's upstream parameters as stored (the input
                the reference's loader.feeds_from_params maps to tiny.npz's feeds).

  qwen35_256_compiled.json.gz  compiled.to_json of the reference's own 256^2
                fp16-weight plan (gzip).

`--quant-only` regenerates quant.npz alone, `--params-only` tiny_params.npz
alone, `--compiled-only` qwen35_256_compiled.json.gz alone.

The fixtures are small (the biggest is well under 2 MB) and are committed;
tests read them without the reference present.
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import hexlib.graph.opdefs  # noqa: F401 -- registers the op kinds
    from hexlib.exec import interpreter
    from hexlib.exec.wholeplan import build_whole_plan_batch
    from hexlib.graph import compiled as compiled_mod
    from hexlib.graph.ops import REGISTRY
    from hexlib.graph.pipeline import compile_model
    from hexlib.models import loader
    from hexlib.models.qwen35 import qwen35_at
    from hexlib.models.vit import VitConfig, build_vision_encoder
    from hexlib.result import Err
    from hexlib.runtime import wire

    tiny = VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                     patch_size=4, temporal_patch_size=2, in_channels=3,
                     spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                     rope_theta=10000.0, image_size=32, act_dtype="fp32",
                     weight_dtype="fp32")
    z = np.load(os.path.join(ref_root, "hexlib", "tests", "data",
                             "qwen35_vision_tiny.npz"))

    # ---- tiny.npz ------------------------------------------------------------
    out = {}
    g32 = build_vision_encoder(tiny)
    feeds = loader.feeds_from_params(g32, tiny, lambda n: z[f"param::{n}"])
    feeds["image"] = z["image"]
    for k, v in feeds.items():
        out[f"feed::{k}"] = np.asarray(v, np.float32)
    out["expected_merged"] = z["expected_merged"]
    out["patches_upstream"] = z["patches_upstream"]
    for act, wdt in (("fp32", "fp32"), ("fp16", "fp16")):
        cfg = dataclasses.replace(tiny, act_dtype=act, weight_dtype=wdt)
        g = build_vision_encoder(cfg)
        m = compile_model(g, budget=1 << 22)
        assert not isinstance(m, Err), m
        f = {}
        for k, v in feeds.items():
            t = g.tensor(k)
            f[k] = np.asarray(v, np.float16).astype(np.float32) if t.dtype == "fp16" else v
        rep = interpreter.run(m, f)
        assert not isinstance(rep, Err), rep
        out[f"interp_{act}_{wdt}"] = rep.outputs[g.outputs[0]]
    np.savez_compressed(os.path.join(HERE, "tiny.npz"), **out)

    # ---- ops.npz ---------------------------------------------------------------
    rng = np.random.default_rng(123)
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)  # noqa: E731
    cases = {}

    def case(name, kind, arrays, attrs):
        (res,) = REGISTRY.get(kind).reference(tuple(arrays), attrs)
        cases[name] = (kind, arrays, attrs, np.asarray(res))

    case("add", "add", [f16(rng.standard_normal((64, 96))), f16(rng.standard_normal((64, 96)))], {})
    case("add_f32", "add", [f16(rng.standard_normal((64, 96))),
                            rng.standard_normal((64, 96)).astype(np.float32) * 0.02], {})
    case("scale", "scale", [f16(rng.standard_normal((4, 64, 32)))], {"factor": 0.125})
    case("layernorm", "layernorm", [f16(rng.standard_normal((16, 768))),
                                    (1 + 0.02 * rng.standard_normal(768)).astype(np.float32),
                                    (0.02 * rng.standard_normal(768)).astype(np.float32)],
         {"eps": 1e-6})
    case("layernorm_c64", "layernorm", [f16(rng.standard_normal((4, 64))),
                                        np.ones(64, np.float32), np.zeros(64, np.float32)],
         {"eps": 1e-6})
    case("gelu_tanh", "gelu_tanh", [f16(rng.standard_normal((8, 256)) * 3)], {})
    case("gelu_erf", "gelu_erf", [f16(rng.standard_normal((8, 256)) * 3)], {})
    sm = f16(rng.standard_normal((3, 8, 64)) * 3)
    sm[0, 0, 5] = 90.0
    case("softmax", "softmax", [sm], {"axis": -1})
    case("matmul", "matmul", [f16(rng.standard_normal((3, 40, 128))),
                              f16(rng.standard_normal((3, 128, 56)) * 0.1)], {})
    for act in ("none", "gelu_tanh", "gelu_erf"):
        case(f"matmul_epilogue_{act}", "matmul_epilogue",
             [f16(rng.standard_normal((20, 128))), f16(rng.standard_normal((128, 96)) * 0.1),
              (0.1 * rng.standard_normal(96)).astype(np.float32)], {"act": act})
    case("cast", "cast", [(rng.standard_normal((33, 17)) * 100).astype(np.float32)],
         {"dtype": "fp16"})
    case("transpose_th", "transpose", [f16(rng.standard_normal((8, 3, 64)))], {"perm": (1, 0, 2)})
    case("transpose_hd", "transpose", [f16(rng.standard_normal((5, 40, 7)))], {"perm": (0, 2, 1)})
    case("patchify", "patchify", [rng.standard_normal((3, 2, 32, 32)).astype(np.float32)],
         {"patch": 4, "temporal_patch": 2, "merge": 2, "grid_h": 8, "grid_w": 8})
    ang = rng.uniform(-3, 3, (6, 64)).astype(np.float32)
    case("rope_2d", "rope_2d", [f16(rng.standard_normal((6, 3, 64))), np.cos(ang), np.sin(ang)], {})
    case("reshape", "reshape", [f16(rng.standard_normal((16, 4, 8)))], {"shape": (16, 32)})
    packed = {}
    meta = {}
    for name, (kind, arrays, attrs, res) in cases.items():
        for i, a in enumerate(arrays):
            packed[f"{name}::in{i}"] = np.asarray(a)
        packed[f"{name}::out"] = res
        meta[name] = {"kind": kind, "n_in": len(arrays),
                      "attrs": {k: (list(v) if isinstance(v, tuple) else v) for k, v in attrs.items()}}
    packed["__meta__"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **packed)

    # ---- plans.json ------------------------------------------------------------------
    plans = {}
    configs = {"tiny_fp16": dataclasses.replace(tiny, act_dtype="fp16", weight_dtype="fp16")}
    for s in (256, 512, 1024):
        configs[f"qwen35_{s}"] = dataclasses.replace(qwen35_at(s), weight_dtype="fp16")
    budgets = {"tiny_fp16": 1 << 22, "qwen35_256": 8 << 20, "qwen35_512": 64 << 20,
               "qwen35_1024": 900 << 20}
    for key, cfg in configs.items():
        g = build_vision_encoder(cfg)
        m = compile_model(g, budget=budgets[key])
        assert not isinstance(m, Err), (key, m)
        plans[key] = {
            "tensors": {n: [t.dtype, list(t.shape), bool(t.const)] for n, t in m.graph.tensors.items()},
            "ops": [[o.id, o.kind, list(o.inputs), list(o.outputs),
                     {k: (list(v) if isinstance(v, tuple) else v) for k, v in o.attrs.items()}]
                    for o in m.graph.ops],
            "inputs": list(m.graph.inputs), "outputs": list(m.graph.outputs),
            "step_order": [s.op.id for s in m.plan.steps if s.op is not None],
            "n_steps": len(m.plan.steps),
            "vtcm_high_water": m.plan.vtcm_high_water,
        }
        if key == "tiny_fp16":
            with open(os.path.join(HERE, "tiny_compiled.json"), "w") as fh:
                fh.write(compiled_mod.to_json(m))
            tiny_m, tiny_cfg16 = m, cfg
    with open(os.path.join(HERE, "plans.json"), "w") as fh:
        json.dump(plans, fh, sort_keys=True, separators=(",", ":"))

    # ---- wire.npz ----------------------------------------------------------------------
    w = {}
    bufs = [wire.BufDesc(fd=3, size=8320), wire.BufDesc(fd=5, size=8320, flags=0)]
    tens = [wire.TensorDesc(0, 0, 4100 * 2, "fp16", "row_major", (4100, 1, 1, 1)),
            wire.TensorDesc(1, 64, 4100 * 2, "fp16", "row_major", (4100, 1, 1, 1))]
    ops = [wire.OpDesc(kind=9, params=(struct.unpack("<i", struct.pack("<f", 0.125))[0],),
                       src=(0,), dst=(1,))]
    w["one_op"] = np.frombuffer(wire.pack_batch(bufs, tens, ops), np.uint8)
    f16feeds = {k: (np.asarray(v, np.float16).astype(np.float32)
                    if tiny_m.graph.tensor(k).dtype == "fp16" else v)
                for k, v in feeds.items() if k in tiny_m.graph.tensors}
    wb = build_whole_plan_batch(tiny_m, f16feeds)
    w["tiny_whole_plan"] = np.frombuffer(wb.blob, np.uint8)
    w["tiny_whole_plan_ops"] = np.frombuffer(json.dumps(list(wb.op_names)).encode(), np.uint8)
    rsp = struct.pack("<IIIIQII", wire.BATCH_MAGIC, wire.BATCH_VERSION, 1, 2, 777, 75, 0)
    rsp += struct.pack("<IIQ", 9, 1, 300) + struct.pack("<IIQ", 5, 13, 0)
    w["response"] = np.frombuffer(rsp, np.uint8)
    np.savez_compressed(os.path.join(HERE, "wire.npz"), **w)

    # ---- tables.npz ----------------------------------------------------------------------
    t = {}
    for key, cfg in (("tiny", tiny), ("qwen35_256", qwen35_at(256))):
        c, s = loader.rope_tables(cfg)
        t[f"{key}::cos"], t[f"{key}::sin"] = c, s
    np.savez_compressed(os.path.join(HERE, "tables.npz"), **t)
    print("wrote", sorted(os.listdir(HERE)))


def make_quant(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import hexlib.graph.opdefs  # noqa: F401
    from hexlib.exec import interpreter
    from hexlib.exec.quant import (dequantize_q4_0, dequantize_q8_0, quantize_q4_0,
                                   quantize_q8_0)
    from hexlib.exec.wholeplan import build_whole_plan_batch
    from hexlib.graph.pipeline import compile_model
    from hexlib.models import loader
    from hexlib.models.vit import VitConfig, build_vision_encoder
    from hexlib.result import Err

    q = {}
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((6, 96)) * np.array([[0.02], [1.0], [3.0], [0.5], [10.0], [1e-3]])
         ).astype(np.float32)
    halves = np.array([-7.5, -6.5, -5.5, -4.5, -3.5, -2.5, -1.5, -0.5,
                       0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5], np.float32)
    edge = np.zeros((4, 96), np.float32)
    edge[0, :32] = np.concatenate([[-8.0], halves, [-8.0], halves])      # q4_0 exact halves
    edge[0, 32:64] = np.linspace(-1, 3, 32)                               # positive extreme
    edge[1, :32] = np.arange(32) - 15.5                                   # q8_0 halves
    edge[1, 32:64] = np.where(np.arange(32) == 5, 1000.0, 1.0)            # extreme, d narrowing
    edge[2, 64:] = np.linspace(-127, 127, 32) * 0.1                       # |q| up to 127
    edge[3, :] = 0.0                                                      # all-zero blocks
    xs = np.concatenate([x, edge]).astype(np.float32)
    q["x"] = xs
    b4, b8 = quantize_q4_0(xs), quantize_q8_0(xs)
    q["q4_0"] = np.frombuffer(b4, np.uint8)
    q["q8_0"] = np.frombuffer(b8, np.uint8)
    q["deq_q4_0"] = dequantize_q4_0(b4, xs.shape)
    q["deq_q8_0"] = dequantize_q8_0(b8, xs.shape)

    tiny = VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                     patch_size=4, temporal_patch_size=2, in_channels=3,
                     spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                     rope_theta=10000.0, image_size=32, act_dtype="fp16",
                     weight_dtype="fp16")
    z = np.load(os.path.join(ref_root, "hexlib", "tests", "data", "qwen35_vision_tiny.npz"))
    g = build_vision_encoder(tiny)
    feeds = loader.feeds_from_params(g, tiny, lambda n: z[f"param::{n}"])
    feeds["image"] = z["image"]
    feeds = {k: (np.asarray(v, np.float16).astype(np.float32)
                 if g.tensor(k).dtype == "fp16" else np.asarray(v, np.float32))
             for k, v in feeds.items()}
    m = compile_model(g, budget=1 << 22)
    assert not isinstance(m, Err), m
    wb = build_whole_plan_batch(m, feeds)
    q["plan_blob"] = np.frombuffer(wb.blob, np.uint8)
    q["plan_payload"] = np.frombuffer(bytes(wb.payload), np.uint8)
    out_name = g.outputs[0]
    po = wb.placements[out_name]
    q["plan_out"] = np.array([po.offset, po.nbytes], np.int64)
    q["plan_out_shape"] = np.array(g.tensor(out_name).shape, np.int64)
    quantized = sorted(n for n, p in wb.placements.items() if p.dtype == "q4_0")
    q["plan_quantized"] = np.frombuffer(json.dumps(quantized).encode(), np.uint8)
    deq = dict(feeds)
    for n in quantized:
        w = np.asarray(feeds[n], np.float32)
        deq[n] = dequantize_q4_0(quantize_q4_0(w), w.shape).astype(np.float16).astype(np.float32)
    rep = interpreter.run(m, deq)
    assert not isinstance(rep, Err), rep
    q["plan_expected"] = np.asarray(rep.outputs[out_name], np.float32)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **q)
    print("wrote quant.npz")


def make_compiled(ref_root: str) -> None:
    """qwen35_256_compiled.json.gz: hexlib.graph.compiled.to_json of the
    reference's own compile_model plan for the 256^2 encoder with fp16
    weights (VTCM budget 8 MiB), gzip-compressed."""
    import gzip
    sys.path.insert(0, ref_root)
    import hexlib.graph.opdefs  # noqa: F401 -- registers the op kinds
    from hexlib.graph import compiled
    from hexlib.graph.pipeline import compile_model
    from hexlib.models.qwen35 import qwen35_at
    from hexlib.models.vit import build_vision_encoder
    from hexlib.result import Err
    cfg = dataclasses.replace(qwen35_at(256), weight_dtype="fp16")
    m = compile_model(build_vision_encoder(cfg), budget=8 << 20)
    assert not isinstance(m, Err), m
    with gzip.open(os.path.join(HERE, "qwen35_256_compiled.json.gz"), "wt") as fh:
        fh.write(compiled.to_json(m))
    print("wrote qwen35_256_compiled.json.gz")


def make_params(ref_root: str) -> None:
    """tiny_params.npz: the upstream (transformers-named) parameters of the
    reference's tiny golden, exactly as stored there -- the input of
    hexlib/models/loader.py feeds_from_params, whose output is tiny.npz's
    feed::* arrays."""
    z = np.load(os.path.join(ref_root, "hexlib", "tests", "data", "qwen35_vision_tiny.npz"))
    params = {k: z[k] for k in z.files if k.startswith("param::")}
    np.savez_compressed(os.path.join(HERE, "tiny_params.npz"), **params)
    print(f"wrote tiny_params.npz ({len(params)} parameters)")


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("HEXLIB_REFERENCE")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/hexlib-checkout "
                 "[--quant-only | --params-only | --compiled-only] (or set HEXLIB_REFERENCE)")
    if "--params-only" in sys.argv:
        make_params(root)
        sys.exit(0)
    if "--compiled-only" in sys.argv:
        make_compiled(root)
        sys.exit(0)
    if "--quant-only" not in sys.argv:
        main(root)
        make_params(root)
        make_compiled(root)
    make_quant(root)
