"""The graph the CUDA path executes: IR, the vision-encoder builder, fusion,
and the rewrites only this backend performs.

The reference's graph compiler is the contract this backend consumes -- its
`Compiled(graph, plan)` is accepted as is by `wholeplan.build_cuda_plan` --
but it is not importable where the backend runs, so the part of it that
decides WHAT executes is restated here, producing the same post-fusion graph
(same tensor names, shapes, dtypes, op ids, kinds and attrs; checked against
the reference by tests/test_graph_matches_reference.py):

  * `Tensor`, `Op`, `Graph`                    hexlib/graph/ir.py:78-225
  * `VitConfig`, `build_vision_encoder`        hexlib/models/vit.py:17-218
  * `QWEN35_08B_VISION`, `qwen35_at`           hexlib/models/qwen35.py:15-52
  * `fuse` (matmul + bias add (+ GELU))        hexlib/graph/fuse.py:16-92
  * `compile_for_cuda` -> `ExecPlan`           the executable half of
                                               hexlib/graph/pipeline.py:59-150

VTCM allocation and DMA insertion are NOT restated: on the GPU the arena is
laid out by `wholeplan`, and tiles move by TMA inside the kernels.

CUDA-ONLY REWRITES (`fuse_attention`, `fuse_residual`) turn chains of plan
ops into the appended wire kinds `attention` and `matmul_epilogue_residual`.
They change which kernels run and how many intermediates are written, not
the function computed; tests compare both forms against the oracle.
"""
from __future__ import annotations

import dataclasses
import json
import math
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Mapping

DTYPES = frozenset({"fp32", "fp16", "int32", "q4_0", "q8_0"})
_DENSE_BYTES = {"fp32": 4, "fp16": 2, "int32": 4}
_BLOCK = {"q4_0": (32, 18), "q8_0": (32, 34)}


def nbytes(shape: tuple[int, ...], dtype: str) -> int:
    """Bytes of a tensor (ir.py:40-56): dense, or 32-element quantized blocks."""
    n = math.prod(shape) if shape else 1
    if dtype in _BLOCK:
        blk, blk_bytes = _BLOCK[dtype]
        if not shape or shape[-1] % blk:
            raise ValueError(f"{dtype} tensor {shape} needs a last dim multiple of {blk}")
        return n // blk * blk_bytes
    if dtype not in _DENSE_BYTES:
        raise ValueError(f"unknown dtype {dtype!r}")
    return n * _DENSE_BYTES[dtype]


@dataclass(frozen=True)
class Tensor:
    name: str
    dtype: str
    shape: tuple[int, ...]
    const: bool = False

    @property
    def nbytes(self) -> int:
        return nbytes(self.shape, self.dtype)


@dataclass(frozen=True)
class Op:
    id: int
    kind: str
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]
    attrs: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        object.__setattr__(self, "inputs", tuple(self.inputs))
        object.__setattr__(self, "outputs", tuple(self.outputs))
        object.__setattr__(self, "attrs", MappingProxyType(dict(self.attrs)))


@dataclass(frozen=True)
class Graph:
    tensors: Mapping[str, Tensor]
    ops: tuple[Op, ...]
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]

    def __post_init__(self) -> None:
        object.__setattr__(self, "tensors", MappingProxyType(dict(self.tensors)))
        object.__setattr__(self, "ops", tuple(self.ops))
        object.__setattr__(self, "inputs", tuple(self.inputs))
        object.__setattr__(self, "outputs", tuple(self.outputs))

    def tensor(self, name: str) -> Tensor:
        return self.tensors[name]

    def problems(self) -> list[str]:
        """Structural problems (ir.py:164-225), as text; empty means valid."""
        out: list[str] = []
        if not self.ops:
            out.append("graph has no ops")
        if not self.outputs:
            out.append("graph declares no outputs")
        written = set(self.inputs) | {n for n, t in self.tensors.items() if t.const}
        seen: set[int] = set()
        for op in self.ops:
            if op.id in seen:
                out.append(f"duplicate op id {op.id}")
            seen.add(op.id)
            for n in op.inputs:
                if n not in self.tensors:
                    out.append(f"op {op.id} ({op.kind}) reads undeclared {n!r}")
                elif n not in written:
                    out.append(f"op {op.id} ({op.kind}) reads {n!r} before it is written")
            for n in op.outputs:
                if n not in self.tensors:
                    out.append(f"op {op.id} ({op.kind}) writes undeclared {n!r}")
                elif n in written:
                    out.append(f"tensor {n!r} is written twice (op {op.id})")
                else:
                    written.add(n)
        for n in self.outputs:
            if n not in written:
                out.append(f"graph output {n!r} is never written")
        return out


# ---- the model ---------------------------------------------------------------

@dataclass(frozen=True)
class VitConfig:
    """vit.py:17-48."""
    depth: int
    hidden_size: int
    num_heads: int
    intermediate_size: int
    patch_size: int
    temporal_patch_size: int
    in_channels: int
    spatial_merge_size: int
    out_hidden_size: int
    layernorm_eps: float
    rope_theta: float
    image_size: int
    act_dtype: str = "fp32"
    weight_dtype: str = "fp32"

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def num_tokens(self) -> int:
        return self.grid * self.grid

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def merge_unit(self) -> int:
        return self.spatial_merge_size ** 2


# qwen35.py:15-42 -- the Qwen3.5-0.8B vision tower. The reference ships it
# with q4_0 weights for the DSP; this backend's configurations use fp16
# weights (weight_dtype="fp16"), the variant `qwen35_at` + replace produces.
QWEN35_08B_VISION = VitConfig(
    depth=12, hidden_size=768, num_heads=12, intermediate_size=3072,
    patch_size=16, temporal_patch_size=2, in_channels=3, spatial_merge_size=2,
    out_hidden_size=1024, layernorm_eps=1e-6, rope_theta=10000.0,
    image_size=256, act_dtype="fp16", weight_dtype="q4_0",
)


def qwen35_at(image_size: int, weight_dtype: str = "fp16",
              act_dtype: str = "fp16") -> VitConfig:
    """The tower at another square resolution (qwen35.py:45-52), fp16 weights
    by default."""
    return dataclasses.replace(QWEN35_08B_VISION, image_size=image_size,
                               weight_dtype=weight_dtype, act_dtype=act_dtype)


def config_problems(cfg: VitConfig) -> list[str]:
    """vit.py:247-283."""
    out = []
    for f in dataclasses.fields(VitConfig):
        v = getattr(cfg, f.name)
        if isinstance(v, int) and not isinstance(v, bool) and v <= 0:
            out.append(f"{f.name} {v} must be positive")
    if out:
        return out
    if cfg.image_size % cfg.patch_size:
        out.append(f"image_size {cfg.image_size} is not divisible by patch_size {cfg.patch_size}")
    elif cfg.grid % cfg.spatial_merge_size:
        out.append(f"patch grid {cfg.grid} is not divisible by spatial_merge_size")
    if cfg.hidden_size % cfg.num_heads:
        out.append("hidden_size is not divisible by num_heads")
    elif cfg.head_dim % 2:
        out.append("head_dim must be even for 2D RoPE")
    return out


class _Builder:
    def __init__(self, cfg: VitConfig) -> None:
        self.cfg = cfg
        self.tensors: dict[str, Tensor] = {}
        self.ops: list[Op] = []

    def declare(self, name, shape, dtype, const=False) -> str:
        if name in self.tensors:
            raise ValueError(f"tensor {name!r} declared twice")
        self.tensors[name] = Tensor(name, dtype, tuple(shape), const)
        return name

    def const(self, name, shape, dtype=None) -> str:
        return self.declare(name, shape, dtype or self.cfg.weight_dtype, const=True)

    def emit(self, kind, inputs, out, shape, attrs=None, dtype=None) -> str:
        self.declare(out, shape, dtype or self.cfg.act_dtype)
        self.ops.append(Op(len(self.ops), kind, tuple(inputs), (out,), attrs or {}))
        return out

    def linear(self, x, wname, bname, k, n, out) -> str:
        """matmul + bias add, weight [k, n], bias fp32 (vit.py:91-96)."""
        w = self.const(wname, (k, n))
        b = self.const(bname, (n,), "fp32")
        rows = self.tensors[x].shape[:-1]
        h = self.emit("matmul", (x, w), f"{out}.mm", rows + (n,))
        return self.emit("add", (h, b), out, rows + (n,))

    def layernorm(self, x, wname, bname, out, shape, eps) -> str:
        w = self.const(wname, (shape[-1],), "fp32")
        b = self.const(bname, (shape[-1],), "fp32")
        return self.emit("layernorm", (x, w, b), out, shape, {"eps": eps})


def build_vision_encoder(cfg: VitConfig) -> Graph:
    """The encoder graph (vit.py:113-218): patchify, cast, patch embed,
    + pos_embed, `depth` pre-LayerNorm blocks with 2D RoPE attention and a
    GELU-tanh MLP, then the 2x2 merger (LayerNorm, reshape, GELU-erf MLP)."""
    problems = config_problems(cfg)
    if problems:
        raise ValueError("invalid vision config: " + "; ".join(problems))
    b = _Builder(cfg)
    n, H = cfg.num_tokens, cfg.hidden_size
    heads, d = cfg.num_heads, cfg.head_dim
    merge = cfg.spatial_merge_size
    feat = cfg.in_channels * cfg.temporal_patch_size * cfg.patch_size ** 2

    image = b.declare("image", (cfg.in_channels, cfg.temporal_patch_size,
                                cfg.image_size, cfg.image_size), "fp32")
    patches = b.emit("patchify", (image,), "patches", (n, feat), {
        "patch": cfg.patch_size, "temporal_patch": cfg.temporal_patch_size,
        "merge": merge, "grid_h": cfg.grid, "grid_w": cfg.grid}, dtype="fp32")
    pc = b.emit("cast", (patches,), "patches.cast", (n, feat),
                {"dtype": cfg.act_dtype}, dtype=cfg.act_dtype)
    emb = b.linear(pc, "w_patch_embed", "b_patch_embed", feat, H, "patch_embed.out")
    pos = b.const("pos_embed", (n, H), "fp32")
    x = b.emit("add", (emb, pos), "x0", (n, H))
    cos = b.const("rope_cos", (n, d), "fp32")
    sin = b.const("rope_sin", (n, d), "fp32")

    for layer in range(cfg.depth):
        p = f"blk{layer}"
        a = b.layernorm(x, f"{p}.ln1_w", f"{p}.ln1_b", f"{p}.ln1.out", (n, H),
                        cfg.layernorm_eps)
        t = {}
        for which in ("q", "k", "v"):
            proj = b.linear(a, f"{p}.w{which}", f"{p}.b{which}", H, H, f"{p}.{which}.out")
            hd = b.emit("reshape", (proj,), f"{p}.{which}.h", (n, heads, d),
                        {"shape": (n, heads, d)})
            if which in ("q", "k"):
                hd = b.emit("rope_2d", (hd, cos, sin), f"{p}.{which}.rope", (n, heads, d))
            t[which] = b.emit("transpose", (hd,), f"{p}.{which}.t", (heads, n, d),
                              {"perm": (1, 0, 2)})
        qs = b.emit("scale", (t["q"],), f"{p}.q.scaled", (heads, n, d),
                    {"factor": float(d) ** -0.5})
        ktt = b.emit("transpose", (t["k"],), f"{p}.k.tt", (heads, d, n), {"perm": (0, 2, 1)})
        s = b.emit("matmul", (qs, ktt), f"{p}.scores", (heads, n, n))
        pr = b.emit("softmax", (s,), f"{p}.probs", (heads, n, n), {"axis": -1})
        ctx = b.emit("matmul", (pr, t["v"]), f"{p}.ctx", (heads, n, d))
        ctxt = b.emit("transpose", (ctx,), f"{p}.ctx.t", (n, heads, d), {"perm": (1, 0, 2)})
        ctxf = b.emit("reshape", (ctxt,), f"{p}.ctx.f", (n, H), {"shape": (n, H)})
        proj = b.linear(ctxf, f"{p}.wo", f"{p}.bo", H, H, f"{p}.o.out")
        xa = b.emit("add", (x, proj), f"{p}.resid1", (n, H))
        c = b.layernorm(xa, f"{p}.ln2_w", f"{p}.ln2_b", f"{p}.ln2.out", (n, H),
                        cfg.layernorm_eps)
        f1 = b.linear(c, f"{p}.w_fc1", f"{p}.b_fc1", H, cfg.intermediate_size, f"{p}.fc1.out")
        g = b.emit("gelu_tanh", (f1,), f"{p}.act", (n, cfg.intermediate_size))
        f2 = b.linear(g, f"{p}.w_fc2", f"{p}.b_fc2", cfg.intermediate_size, H, f"{p}.fc2.out")
        x = b.emit("add", (xa, f2), f"{p}.resid2", (n, H))

    M = H * cfg.merge_unit
    mn = b.layernorm(x, "m_ln_w", "m_ln_b", "merger.ln.out", (n, H), cfg.layernorm_eps)
    mc = b.emit("reshape", (mn,), "merger.concat", (n // cfg.merge_unit, M),
                {"shape": (n // cfg.merge_unit, M)})
    m1 = b.linear(mc, "w_m1", "b_m1", M, M, "merger.fc1.out")
    mg = b.emit("gelu_erf", (m1,), "merger.act", (n // cfg.merge_unit, M))
    out = b.linear(mg, "w_m2", "b_m2", M, cfg.out_hidden_size, "merger.out")
    return Graph(b.tensors, tuple(b.ops), (image,), (out,))


def weight_names(cfg: VitConfig) -> tuple[str, ...]:
    """Every const the graph needs, sorted (vit.py:99-110)."""
    g = build_vision_encoder(cfg)
    return tuple(sorted(n for n, t in g.tensors.items() if t.const))


# ---- passes ------------------------------------------------------------------------

FUSABLE_ACTS = ("gelu_tanh", "gelu_erf")


def _consumers(graph: Graph) -> dict[str, list[Op]]:
    out: dict[str, list[Op]] = {}
    for op in graph.ops:
        for n in op.inputs:
            out.setdefault(n, []).append(op)
    return out


def fuse(graph: Graph) -> Graph:
    """Fold `add(matmul, const 1-D bias)` and an optional GELU after it into
    one `matmul_epilogue` with attr `act` (fuse.py:16-92). The matmul's and
    the add's intermediates must each have exactly one consumer and not be
    graph outputs; the fused op keeps the matmul's id."""
    cons = _consumers(graph)
    protected = set(graph.outputs)

    def only(name: str, skip: set[int]) -> Op | None:
        if name in protected:
            return None
        found = [o for o in cons.get(name, []) if o.id not in skip]
        return found[0] if len(found) == 1 and len(cons.get(name, [])) == 1 else None

    consumed: set[int] = set()
    rewritten: dict[int, Op] = {}
    dropped: set[str] = set()
    for op in graph.ops:
        if op.id in consumed or op.kind != "matmul":
            continue
        mm = op.outputs[0]
        add = only(mm, consumed)
        if add is None or add.kind != "add" or len(add.inputs) != 2:
            continue
        bias = add.inputs[1] if add.inputs[0] == mm else add.inputs[0]
        bt = graph.tensors.get(bias)
        if bt is None or not bt.const or len(bt.shape) != 1:
            continue
        act, tail = "none", add
        a = only(add.outputs[0], consumed | {add.id})
        if a is not None and a.kind in FUSABLE_ACTS:
            act, tail = a.kind, a
        rewritten[op.id] = Op(op.id, "matmul_epilogue", (op.inputs[0], op.inputs[1], bias),
                              tail.outputs, {"act": act})
        consumed.add(add.id)
        dropped.add(mm)
        if tail is not add:
            consumed.add(tail.id)
            dropped.add(add.outputs[0])
    if not rewritten:
        return graph
    ops = tuple(rewritten.get(o.id, o) for o in graph.ops if o.id not in consumed)
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    return Graph(tensors, ops, graph.inputs, graph.outputs)


def fuse_attention(graph: Graph) -> Graph:
    """CUDA-only: scale(q) -> matmul(., transpose_hd(k)) -> softmax -> matmul(., v)
    becomes one `attention(q, k, v)` op with attr `scale`, and the [H, T, T]
    scores and probabilities are never written. Each removed intermediate must
    have exactly one consumer and not be a graph output."""
    cons = _consumers(graph)
    protected = set(graph.outputs)
    producer = {o.outputs[0]: o for o in graph.ops}

    def sole(name):
        c = cons.get(name, [])
        return c[0] if len(c) == 1 and name not in protected else None

    consumed: set[int] = set()
    rewritten: dict[int, Op] = {}
    dropped: set[str] = set()
    for sm in graph.ops:
        if sm.kind != "softmax" or sm.attrs.get("axis") != -1:
            continue
        qk = producer.get(sm.inputs[0])
        pv = sole(sm.outputs[0])
        if qk is None or qk.kind != "matmul" or pv is None or pv.kind != "matmul":
            continue
        if pv.inputs[0] != sm.outputs[0] or sole(qk.outputs[0]) is not sm:
            continue
        sc = producer.get(qk.inputs[0])
        kt = producer.get(qk.inputs[1])
        if sc is None or sc.kind != "scale" or kt is None or kt.kind != "transpose":
            continue
        if tuple(kt.attrs.get("perm", ())) != (0, 2, 1):
            continue
        if sole(sc.outputs[0]) is not qk or sole(kt.outputs[0]) is not qk:
            continue
        q, k, v = sc.inputs[0], kt.inputs[0], pv.inputs[1]
        shp = graph.tensors[q].shape
        if len(shp) != 3 or graph.tensors[k].shape != shp or graph.tensors[v].shape != shp:
            continue
        if not all(graph.tensors[n].dtype == "fp16" for n in (q, k, v, pv.outputs[0])):
            continue
        rewritten[pv.id] = Op(pv.id, "attention", (q, k, v), pv.outputs,
                              {"scale": float(sc.attrs["factor"])})
        consumed |= {sc.id, kt.id, qk.id, sm.id}
        dropped |= {sc.outputs[0], kt.outputs[0], qk.outputs[0], sm.outputs[0]}
    if not rewritten:
        return graph
    ops = tuple(rewritten.get(o.id, o) for o in graph.ops if o.id not in consumed)
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    return Graph(tensors, ops, graph.inputs, graph.outputs)


def fuse_residual(graph: Graph) -> Graph:
    """CUDA-only: `add(r, matmul_epilogue(a, w, b))` whose matmul result has
    no other consumer becomes `matmul_epilogue_residual(a, w, b, r)`; the
    epilogue rounds the product to fp16 before adding, as the two ops do."""
    cons = _consumers(graph)
    protected = set(graph.outputs)
    producer = {o.outputs[0]: o for o in graph.ops}
    consumed: set[int] = set()
    rewritten: dict[int, Op] = {}
    dropped: set[str] = set()
    for add in graph.ops:
        if add.kind != "add" or len(add.inputs) != 2:
            continue
        for side in (1, 0):
            mm = producer.get(add.inputs[side])
            r = add.inputs[1 - side]
            if mm is None or mm.kind != "matmul_epilogue" or mm.id in consumed:
                continue
            out = mm.outputs[0]
            if out in protected or len(cons.get(out, [])) != 1:
                continue
            rt, ot = graph.tensors[r], graph.tensors[out]
            if rt.shape != ot.shape or rt.dtype != "fp16" or ot.dtype != "fp16" or rt.const:
                continue
            if graph.tensors[add.outputs[0]].dtype != "fp16":
                continue
            rewritten[add.id] = Op(add.id, "matmul_epilogue_residual",
                                   tuple(mm.inputs) + (r,), add.outputs,
                                   {"act": mm.attrs.get("act", "none")})
            consumed.add(mm.id)
            dropped.add(out)
            break
    if not rewritten:
        return graph
    # the fused op takes the matmul's place in the order (its inputs are ready there)
    ops = []
    for o in graph.ops:
        if o.id in consumed:
            continue
        ops.append(rewritten.get(o.id, o))
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    return Graph(tensors, tuple(ops), graph.inputs, graph.outputs)


def fuse_patchify_cast(graph: Graph) -> Graph:
    """CUDA-only: `cast(patchify(image), fp16)` whose fp32 patch rows have no
    other consumer becomes one `patchify_cast(image)` writing the fp16 rows
    (each value rounded to nearest even, as the cast rounds it): one pass
    over the image instead of a write and a re-read of the fp32 rows."""
    cons = _consumers(graph)
    protected = set(graph.outputs)
    T = graph.tensors
    rewritten: dict[int, Op] = {}
    consumed: set[int] = set()
    dropped: set[str] = set()
    for pt in graph.ops:
        if pt.kind != "patchify":
            continue
        rows = pt.outputs[0]
        users = cons.get(rows, [])
        if rows in protected or len(users) != 1:
            continue
        cast = users[0]
        if cast.kind != "cast" or cast.attrs.get("dtype") != "fp16" or T[rows].dtype != "fp32":
            continue
        rewritten[pt.id] = Op(pt.id, "patchify_cast", pt.inputs, cast.outputs, dict(pt.attrs))
        consumed.add(cast.id)
        dropped.add(rows)
    if not rewritten:
        return graph
    ops = tuple(rewritten.get(o.id, o) for o in graph.ops if o.id not in consumed)
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    return Graph(tensors, ops, graph.inputs, graph.outputs)


def fold_layernorm(graph: Graph, derived_in: Mapping[str, tuple] | None = None
                   ) -> tuple[Graph, dict[str, tuple]]:
    """CUDA-only, after `fuse_qkv`: a `layernorm(x, gamma, beta)` whose only
    consumer is a GEMM over its output with an fp16 weight W [K, N], N a
    multiple of 256, becomes

        stats = ln_stats(x)                                   [T, 2] fp32
        out   = matmul_epilogue_ln(x, W', cols, stats)         (or ..._ln_rope)

    with W' = fp16(diag(gamma) W) and cols [2, N] = (beta @ W + b; the column
    sums of W') new consts: the GEMM's epilogue forms
    act(rstd * (x @ W' - mean * colsum) + bias) = act(LayerNorm(x) @ W + b),
    so the normalised rows are never written out and read back. The RoPE
    variant takes the two segment tables interleaved ([2T, 2, 16]). New
    consts come back as `{name: (recipe, parts, arg)}` for the batch builder."""
    cons = _consumers(graph)
    protected = set(graph.outputs)
    T = graph.tensors
    rewritten: dict[int, Op] = {}
    new_tensors: dict[str, Tensor] = {}
    dropped: set[str] = set()
    derived: dict[str, tuple] = {}
    for ln in graph.ops:
        if ln.kind != "layernorm" or len(ln.inputs) != 3:
            continue
        y = ln.outputs[0]
        users = cons.get(y, [])
        if y in protected or len(users) != 1:
            continue
        mm = users[0]
        if mm.kind not in ("matmul_epilogue", "matmul_epilogue_rope") or mm.inputs[0] != y:
            continue
        x, gamma, beta = ln.inputs
        w, b = mm.inputs[1], mm.inputs[2]
        wt, bt, xt = T[w], T[b], T[x]
        if not (wt.const and wt.dtype == "fp16" and len(wt.shape) == 2 and bt.const and
                bt.dtype == "fp32" and T[gamma].const and T[beta].const and
                T[gamma].dtype == "fp32" and T[beta].dtype == "fp32"):
            continue
        K, N = wt.shape
        if N % 256 or len(xt.shape) != 2 or xt.shape[1] != K or xt.dtype != "fp16":
            continue
        rope_src = None
        if mm.kind == "matmul_epilogue_rope":
            rec = (derived_in or {}).get(mm.inputs[3])
            if rec is None or rec[0] != "rope_segments":
                continue
            rope_src = tuple(rec[1])
        n_tok = xt.shape[0]
        wf = f"lnfold_w({gamma},{w})"
        cols = f"lnfold_cols({gamma},{beta},{w},{b})"
        stats = f"{y}+stats"
        new_tensors[wf] = Tensor(wf, "fp16", (K, N), True)
        new_tensors[cols] = Tensor(cols, "fp32", (2, N), True)
        new_tensors[stats] = Tensor(stats, "fp32", (n_tok, 2), False)
        derived[wf] = ("ln_fold_w", (gamma, w), 0)
        derived[cols] = ("ln_fold_cols", (gamma, beta, w, b), 0)
        rewritten[ln.id] = Op(ln.id, "ln_stats", (x,), (stats,), {"eps": float(ln.attrs["eps"])})
        act = {"act": mm.attrs.get("act", "none")}
        if mm.kind == "matmul_epilogue":
            rewritten[mm.id] = Op(mm.id, "matmul_epilogue_ln", (x, wf, cols, stats),
                                  mm.outputs, act)
        else:
            seg_cos, seg_idx = mm.inputs[3], mm.inputs[5]
            cos, sin = rope_src
            segtab = f"rope_segtab({cos},{sin})"
            new_tensors[segtab] = Tensor(segtab, "fp32", (T[seg_cos].shape[0], 2, 16), True)
            derived[segtab] = ("rope_segtab", (cos, sin), 0)
            rewritten[mm.id] = Op(mm.id, "matmul_epilogue_ln_rope",
                                  (x, wf, cols, stats, segtab, seg_idx), mm.outputs,
                                  dict(act, rope_cols=int(mm.attrs["rope_cols"])))
        dropped.add(y)
    if not rewritten:
        return graph, {}
    ops = tuple(rewritten.get(o.id, o) for o in graph.ops)
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    tensors.update(new_tensors)
    used = {n for o in ops for n in o.inputs}
    tensors = {n: t for n, t in tensors.items() if not (t.const and n not in used)}
    return Graph(tensors, ops, graph.inputs, graph.outputs), derived


def fuse_qkv(graph: Graph, rope_epilogue: bool = False) -> tuple[Graph, dict[str, tuple]]:
    """CUDA-only, after `fuse_attention`: per block, the q, k and v projections
    (three matmul_epilogue over one input), their reshapes to [T, H, D], the
    rope_2d of q and k, the three [T,H,D] -> [H,T,D] transposes into the
    attention op and the transpose of its output back to [T, H, D] become

        raw   = matmul_epilogue(a, [wq|wk|wv], [bq|bk|bv])   [T, 3, H, D]
        qkv   = rope_qk(raw, cos, sin)                       [T, 3, H, D]  (in place)
        ctx.t = attention_qkv(qkv)                           [T, H, D]

    or, with `rope_epilogue` and an fp16 weight, the rotation applied by the
    GEMM's epilogue before the one fp16 store:

        qkv   = matmul_epilogue_rope(a, [wq|wk|wv], [bq|bk|bv],
                                     seg_cos, seg_sin, seg_idx)  [T, 3, H, D]
        ctx.t = attention_qkv(qkv)

    where seg_cos / seg_sin [2T, 16] and seg_idx [T, 2] int32 are the
    half-symmetric cos/sin tables cut into 16-wide segments and deduplicated
    (a 2-D RoPE repeats each segment across a row or column of the patch
    grid, so the distinct ones are few and stay cache-resident under the
    epilogue); the batch builder refuses tables that are not half-symmetric.

    The concatenated weight and bias and the segment tables are new consts,
    returned as `{name: ("concat", (parts...), axis)}` and
    `{name: ("rope_segments", (cos, sin), which)}` for the batch builder to
    derive from the feeds. Every removed intermediate must have exactly one
    consumer and not be a graph output; anything else leaves the block as it
    was."""
    cons = _consumers(graph)
    protected = set(graph.outputs)
    producer = {o.outputs[0]: o for o in graph.ops}
    T = graph.tensors

    def sole_user(name):
        c = cons.get(name, [])
        return c[0] if len(c) == 1 and name not in protected else None

    def prod(name, kind):
        o = producer.get(name)
        return o if o is not None and o.kind == kind and sole_user(name) is not None else None

    consumed: set[int] = set()
    rewritten: dict[int, Op] = {}
    new_tensors: dict[str, Tensor] = {}
    dropped: set[str] = set()
    derived: dict[str, tuple] = {}
    for att in graph.ops:
        if att.kind != "attention":
            continue
        chain = {}
        ok = True
        for which, name, roped in (("q", att.inputs[0], True), ("k", att.inputs[1], True),
                                   ("v", att.inputs[2], False)):
            tr = prod(name, "transpose")
            if tr is None or tuple(tr.attrs.get("perm", ())) != (1, 0, 2):
                ok = False
                break
            rp = prod(tr.inputs[0], "rope_2d") if roped else None
            if roped and rp is None:
                ok = False
                break
            rs = prod((rp.inputs[0] if roped else tr.inputs[0]), "reshape")
            mm = prod(rs.inputs[0], "matmul_epilogue") if rs is not None else None
            if mm is None or mm.attrs.get("act", "none") != "none":
                ok = False
                break
            chain[which] = (tr, rp, rs, mm)
        if not ok:
            continue
        ctx_t = sole_user(att.outputs[0])
        if ctx_t is None or ctx_t.kind != "transpose" or tuple(ctx_t.attrs.get("perm", ())) != (1, 0, 2):
            continue
        mms = [chain[w][3] for w in "qkv"]
        a = mms[0].inputs[0]
        if any(m.inputs[0] != a for m in mms):
            continue
        rq, rk = chain["q"][1], chain["k"][1]
        if rq.inputs[1:] != rk.inputs[1:]:
            continue
        cos, sin = rq.inputs[1], rq.inputs[2]
        ws = [m.inputs[1] for m in mms]
        bs = [m.inputs[2] for m in mms]
        wdt = T[ws[0]].dtype
        if wdt not in ("fp16", "q4_0", "q8_0") or not all(
                T[w].const and T[w].dtype == wdt and len(T[w].shape) == 2 for w in ws):
            continue
        if not all(T[b].const and T[b].dtype == "fp32" for b in bs):
            continue
        n_tok, heads, d = T[att.outputs[0]].shape[1], T[att.outputs[0]].shape[0], T[att.outputs[0]].shape[2]
        K = T[ws[0]].shape[0]
        if any(T[w].shape != (K, heads * d) for w in ws) or T[a].shape != (n_tok, K) or d != 64:
            continue
        wname = f"concat({ws[0]},{ws[1]},{ws[2]})"
        bname = f"concat({bs[0]},{bs[1]},{bs[2]})"
        raw = f"{mms[0].outputs[0]}+qkv.raw"
        qkv = f"{mms[0].outputs[0]}+qkv"
        new_tensors[wname] = Tensor(wname, wdt, (K, 3 * heads * d), True)
        new_tensors[bname] = Tensor(bname, "fp32", (3 * heads * d,), True)
        new_tensors[raw] = Tensor(raw, "fp16", (n_tok, 3, heads, d), False)
        new_tensors[qkv] = Tensor(qkv, "fp16", (n_tok, 3, heads, d), False)
        derived[wname] = ("concat", tuple(ws), 1)
        derived[bname] = ("concat", tuple(bs), 0)
        if rope_epilogue and wdt == "fp16":
            segs = tuple(f"rope_segments({cos},{sin}).{w}" for w in ("cos", "sin", "idx"))
            new_tensors[segs[0]] = Tensor(segs[0], "fp32", (2 * n_tok, 16), True)
            new_tensors[segs[1]] = Tensor(segs[1], "fp32", (2 * n_tok, 16), True)
            new_tensors[segs[2]] = Tensor(segs[2], "int32", (n_tok, 2), True)
            for i, sname in enumerate(segs):
                derived[sname] = ("rope_segments", (cos, sin), i)
            del new_tensors[raw]
            rewritten[mms[0].id] = Op(mms[0].id, "matmul_epilogue_rope",
                                      (a, wname, bname) + segs, (qkv,),
                                      {"act": "none", "rope_cols": 2 * heads * d})
        else:
            rewritten[mms[0].id] = Op(mms[0].id, "matmul_epilogue", (a, wname, bname), (raw,),
                                      {"act": "none"})
            # the rope takes the k projection's op id, free once that op is gone
            rewritten[mms[1].id] = Op(mms[1].id, "rope_qk", (raw, cos, sin), (qkv,), {})
        rewritten[ctx_t.id] = Op(ctx_t.id, "attention_qkv", (qkv,), ctx_t.outputs,
                                 {"scale": float(att.attrs["scale"])})
        for w in "qkv":
            tr, rp, rs, mm = chain[w]
            for o in (tr, rp, rs, mm):
                if o is not None:
                    consumed.add(o.id)
                    dropped.add(o.outputs[0])
        consumed.add(att.id)
        dropped.add(att.outputs[0])
        consumed.discard(mms[0].id)
        if mms[1].id in rewritten:
            consumed.discard(mms[1].id)
    if not rewritten:
        return graph, {}
    ops = tuple(rewritten.get(o.id, o) for o in graph.ops
                if o.id not in consumed or o.id in rewritten)
    tensors = {n: t for n, t in graph.tensors.items() if n not in dropped}
    tensors.update(new_tensors)
    used = {n for o in ops for n in o.inputs}
    tensors = {n: t for n, t in tensors.items()
               if not (t.const and n not in used)}
    return Graph(tensors, ops, graph.inputs, graph.outputs), derived


# ---- the executable plan -------------------------------------------------------------

@dataclass(frozen=True)
class Step:
    op: Op


@dataclass(frozen=True)
class ExecPlan:
    """What the CUDA path executes: the post-fusion graph and its op order.
    Shaped like the reference's `Compiled(graph, plan)` (compiled.py:33-66)
    where the batch builder reads it: `.graph` and `.plan.steps[i].op`.
    `derived` names consts a rewrite created, with the recipe that builds
    each from the feeds or from other derived consts (`("concat", parts,
    axis)`, `("rope_segments", (cos, sin), which)`, `("rope_segtab", (cos,
    sin), 0)`, `("ln_fold_w", (gamma, w), 0)`, `("ln_fold_cols", (gamma,
    beta, w, b), 0)`)."""
    graph: Graph
    plan: "ExecSteps"
    derived: Mapping[str, tuple] = field(default_factory=dict)


@dataclass(frozen=True)
class ExecSteps:
    steps: tuple[Step, ...]
    target: str = "b200"


def _apply_rewrites(g: Graph, attention: bool, residual: bool, qkv: bool,
                    rope_epilogue: bool = False, ln_fold: bool = False,
                    patch_cast: bool = False):
    derived: dict[str, tuple] = {}
    if patch_cast:
        g = fuse_patchify_cast(g)
    if attention or qkv:
        g = fuse_attention(g)
    if qkv:
        g, derived = fuse_qkv(g, rope_epilogue)
    if ln_fold:
        g, more = fold_layernorm(g, derived)
        derived = {**derived, **more}
    if residual:
        g = fuse_residual(g)
    problems = g.problems()
    if problems:
        raise ValueError("rewritten graph is invalid: " + "; ".join(problems[:5]))
    return g, derived


# The CUDA-only rewrites the encoder runs with unless told otherwise -- the
# plan bench.py measures: fused attention over one packed q/k/v projection
# with RoPE in that GEMM's epilogue, residual adds in the GEMM epilogues,
# patchify writing fp16 rows. (`ln_fold` stays off: measured slower.)
DEFAULT_REWRITES = MappingProxyType({"attention": True, "qkv": True, "rope_epilogue": True,
                                     "residual": True, "patch_cast": True})


def compile_for_cuda(graph: Graph, attention: bool = False, residual: bool = False,
                     qkv: bool = False, rope_epilogue: bool = False,
                     ln_fold: bool = False, patch_cast: bool = False) -> ExecPlan:
    """Fuse (as the reference pipeline does), optionally apply the CUDA-only
    rewrites, and order the ops for execution (the builder's order is
    topological; every rewrite keeps it so). `qkv` implies `attention`;
    `rope_epilogue` moves the packed path's RoPE into the qkv GEMM;
    `ln_fold` folds each layernorm that feeds one GEMM into that GEMM;
    `patch_cast` writes the patch rows as fp16 straight from patchify."""
    problems = graph.problems()
    if problems:
        raise ValueError("graph is structurally invalid: " + "; ".join(problems[:5]))
    g, derived = _apply_rewrites(fuse(graph), attention, residual, qkv, rope_epilogue,
                                 ln_fold, patch_cast)
    return ExecPlan(g, ExecSteps(tuple(Step(o) for o in g.ops)), derived)


def rewrite_compiled(compiled, attention: bool = False, residual: bool = False,
                     qkv: bool = False, rope_epilogue: bool = False,
                     ln_fold: bool = False, patch_cast: bool = False) -> ExecPlan:
    """Apply the CUDA-only rewrites to any compiled pair -- the reference's
    own `Compiled` included -- keeping its plan order for the ops that stay."""
    graph = as_graph(compiled.graph)
    order = [s.op.id for s in compiled.plan.steps if getattr(s, "op", None) is not None]
    by_id = {o.id: o for o in graph.ops}
    g = Graph(graph.tensors, tuple(by_id[i] for i in order), graph.inputs, graph.outputs)
    g, derived = _apply_rewrites(g, attention, residual, qkv, rope_epilogue, ln_fold,
                                 patch_cast)
    return ExecPlan(g, ExecSteps(tuple(Step(o) for o in g.ops)), derived)


def as_graph(g) -> Graph:
    """Convert any graph with the reference's attribute names to ours."""
    if isinstance(g, Graph):
        return g
    tensors = {n: Tensor(t.name, t.dtype, tuple(t.shape), bool(t.const))
               for n, t in g.tensors.items()}
    ops = tuple(Op(o.id, o.kind, tuple(o.inputs), tuple(o.outputs), dict(o.attrs))
                for o in g.ops)
    return Graph(tensors, ops, tuple(g.inputs), tuple(g.outputs))


def _tuples(x):
    if isinstance(x, list):
        return tuple(_tuples(v) for v in x)
    if isinstance(x, dict):
        return {k: _tuples(v) for k, v in x.items()}
    return x


def from_compiled_json(text: str) -> ExecPlan:
    """Load the reference's `Compiled` JSON artefact (compiled.py:72-168):
    the post-fusion graph plus the plan's step order. VTCM slots and DMA
    transfers are read past -- the CUDA arena is laid out by wholeplan."""
    raw = json.loads(text)
    if not isinstance(raw, dict) or "graph" not in raw or "plan" not in raw:
        raise ValueError("not a compiled artefact: needs 'graph' and 'plan'")
    gr = raw["graph"]
    tensors = {t["name"]: Tensor(t["name"], t["dtype"], tuple(t["shape"]),
                                 bool(t.get("const", False))) for t in gr["tensors"]}
    ops = {o["id"]: Op(o["id"], o["kind"], tuple(o["inputs"]), tuple(o["outputs"]),
                       _tuples(o.get("attrs", {}))) for o in gr["ops"]}
    order = []
    for s in raw["plan"]["steps"]:
        op = s.get("op")
        if op is not None:
            order.append(op["id"])
    g = Graph(tensors, tuple(ops[i] for i in order), tuple(gr["inputs"]), tuple(gr["outputs"]))
    return ExecPlan(g, ExecSteps(tuple(Step(o) for o in g.ops)))
