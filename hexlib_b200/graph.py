"""The graph the CUDA path executes: a small IR, the vision encoder written as
a program text for it, the matmul-epilogue fusion, and the rewrites only this
backend performs.

The reference's graph compiler is the contract this backend consumes -- its
`Compiled(graph, plan)` is accepted as is by `wholeplan.build_cuda_plan`, and
its JSON artefact by `from_compiled_json` -- but it is not importable where
the backend runs, so this module produces the same post-fusion graph on its
own: the same tensor names, shapes, dtypes and const flags, op ids, kinds,
inputs, outputs and attrs as hexlib/models/vit.py:113-218 after
hexlib/graph/fuse.py:16-92 (checked against the reference's own plans by
tests/test_graph_matches_reference.py). Those names, ids and attrs are the
interface -- feeds, plans and blobs key on them -- so they are reproduced
exactly; how they are produced is this module's own:

  * the encoder is data: three op programs (stem, block, merger) in a line
    format parsed by `_Program` -- one op per line, consts declared where
    they are first read, shapes and attrs in symbols of the configuration;
  * every graph rewrite, the reference's fusion included, is a set of edits
    recorded on an `_Edit` (replace an op in place, drop ops and tensors, add
    tensors) and applied in one step.

VTCM allocation and DMA insertion are not produced: on the GPU the arena is
laid out by `wholeplan`, and tiles move by TMA inside the kernels.

CUDA-ONLY REWRITES (`fuse_attention`, `fuse_residual`, `fuse_qkv`,
`fuse_patchify_cast`, `fold_layernorm`) turn chains of plan ops into the
appended wire kinds. They change which kernels run and how many
intermediates are written, not the function computed; tests compare both
forms against the oracle.
"""
from __future__ import annotations

import ast
import dataclasses
import json
import re
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Iterable, Mapping

from hexlib_b200 import quant as _quant

DTYPES = frozenset({"fp32", "fp16", "int32", "q4_0", "q8_0"})
_ITEM_BYTES = {"fp32": 4, "fp16": 2, "int32": 4}


def nbytes(shape: tuple[int, ...], dtype: str) -> int:
    """Storage bytes of a tensor: dense element bytes, or 32-element blocks of
    18 (q4_0) / 34 (q8_0) bytes along the last axis (hexlib/graph/ir.py:23-56)."""
    if dtype in _quant.BLOCK_BYTES:
        return _quant.nbytes(tuple(shape), dtype)
    try:
        item = _ITEM_BYTES[dtype]
    except KeyError:
        raise ValueError(f"unknown dtype {dtype!r}") from None
    count = 1
    for d in shape:
        count *= int(d)
    return count * item


# ---- IR ------------------------------------------------------------------------------

@dataclass(frozen=True)
class Tensor:
    """A named value: graph input, intermediate, or const (a weight or table
    fed once per session)."""
    name: str
    dtype: str
    shape: tuple[int, ...]
    const: bool = False

    @property
    def nbytes(self) -> int:
        return nbytes(self.shape, self.dtype)


def _frozen(attrs: Mapping[str, Any]) -> Mapping[str, Any]:
    return MappingProxyType(dict(attrs))


@dataclass(frozen=True)
class Op:
    """One step: `kind` reads `inputs` and writes `outputs` (tensor names)."""
    id: int
    kind: str
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]
    attrs: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        object.__setattr__(self, "inputs", tuple(self.inputs))
        object.__setattr__(self, "outputs", tuple(self.outputs))
        object.__setattr__(self, "attrs", _frozen(self.attrs))

    def with_(self, **changes) -> "Op":
        return dataclasses.replace(self, **changes)


@dataclass(frozen=True)
class Graph:
    """Tensors by name, ops in execution order, graph inputs and outputs."""
    tensors: Mapping[str, Tensor]
    ops: tuple[Op, ...]
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]

    def __post_init__(self) -> None:
        object.__setattr__(self, "tensors", _frozen(self.tensors))
        object.__setattr__(self, "ops", tuple(self.ops))
        object.__setattr__(self, "inputs", tuple(self.inputs))
        object.__setattr__(self, "outputs", tuple(self.outputs))

    def tensor(self, name: str) -> Tensor:
        return self.tensors[name]

    def problems(self) -> list[str]:
        """Why this graph cannot run in its op order (empty when it can): an
        empty graph, an unknown name, a read before any write, a second
        write, a duplicate op id, an output nobody writes. The checks of
        hexlib/graph/ir.py:164-225, as a replay of the op order."""
        issues: list[str] = []
        if not self.ops:
            issues.append("the graph has no ops")
        if not self.outputs:
            issues.append("the graph names no outputs")
        ready = {n for n, t in self.tensors.items() if t.const}
        ready.update(self.inputs)
        ids: set[int] = set()
        for op in self.ops:
            where = f"op {op.id} ({op.kind})"
            if op.id in ids:
                issues.append(f"{where}: its id is used twice")
            ids.add(op.id)
            for name in op.inputs:
                if name not in self.tensors:
                    issues.append(f"{where}: reads {name!r}, which is not declared")
                elif name not in ready:
                    issues.append(f"{where}: reads {name!r} before anything writes it")
            for name in op.outputs:
                if name not in self.tensors:
                    issues.append(f"{where}: writes {name!r}, which is not declared")
                elif name in ready:
                    issues.append(f"{where}: writes {name!r}, which already has a value")
                ready.add(name)
        issues.extend(f"graph output {n!r}: nothing writes it"
                      for n in self.outputs if n not in ready)
        return issues


# ---- the model: configuration ---------------------------------------------------------

@dataclass(frozen=True)
class VitConfig:
    """The vision tower's hyper-parameters, with the field names of
    hexlib/models/vit.py:17-48 (the reference's configs are built from them)."""
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
        """Patches along each side of the image."""
        return self.image_size // self.patch_size

    @property
    def num_tokens(self) -> int:
        return self.grid ** 2

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


# The Qwen3.5-0.8B vision tower (hexlib/models/qwen35.py:15-42): 12 blocks of
# width 768 with 12 heads, MLP 3072, 16x16 patches over 2 frames, 2x2 merge
# to 1024 outputs. The reference ships it with q4_0 weights for the DSP; this
# backend's configurations use fp16 weights (`qwen35_at`'s default).
QWEN35_08B_VISION = VitConfig(
    depth=12, hidden_size=768, num_heads=12, intermediate_size=3072,
    patch_size=16, temporal_patch_size=2, in_channels=3, spatial_merge_size=2,
    out_hidden_size=1024, layernorm_eps=1e-6, rope_theta=10000.0,
    image_size=256, act_dtype="fp16", weight_dtype="q4_0",
)


def qwen35_at(image_size: int, weight_dtype: str = "fp16",
              act_dtype: str = "fp16") -> VitConfig:
    """The tower at another square resolution (hexlib/models/qwen35.py:45-52),
    fp16 weights unless asked otherwise."""
    return dataclasses.replace(QWEN35_08B_VISION, image_size=image_size,
                               weight_dtype=weight_dtype, act_dtype=act_dtype)


def config_problems(cfg: VitConfig) -> list[str]:
    """Why `cfg` cannot describe an encoder (empty when it can): every count
    positive, whole patches, a patch grid the merge divides, whole heads of
    even width (the rotation pairs dimensions) -- the conditions of
    hexlib/models/vit.py:247-283."""
    counts = ("depth", "hidden_size", "num_heads", "intermediate_size", "patch_size",
              "temporal_patch_size", "in_channels", "spatial_merge_size",
              "out_hidden_size", "image_size")
    bad = [f"{k} must be a positive integer, not {getattr(cfg, k)!r}"
           for k in counts if not isinstance(getattr(cfg, k), int) or getattr(cfg, k) <= 0]
    if bad:
        return bad
    if cfg.image_size % cfg.patch_size:
        bad.append(f"a {cfg.image_size}-pixel image is not a whole number of "
                   f"{cfg.patch_size}-pixel patches")
    elif cfg.grid % cfg.spatial_merge_size:
        bad.append(f"the {cfg.grid}-patch grid does not split into "
                   f"{cfg.spatial_merge_size}x{cfg.spatial_merge_size} merge blocks")
    if cfg.hidden_size % cfg.num_heads:
        bad.append(f"width {cfg.hidden_size} does not split into {cfg.num_heads} heads")
    elif cfg.head_dim % 2:
        bad.append(f"head width {cfg.head_dim} is odd; the 2-D rotation needs pairs")
    return bad


# ---- the model: op programs -----------------------------------------------------------
#
# One op per line:   OUT[:dtype] = KIND(ARG, ARG, ...) [SHAPE] key=value ...
#   ARG is a tensor name, or `$name:dtype[SHAPE]` for a const, declared where
#   it is first read (a later `$` of the same name must agree). dtype `w` is
#   the configuration's weight dtype, `act` its activation dtype (the default
#   for outputs). SHAPE and attr values use the symbols `_symbols` defines;
#   `{b}` and `{x}` are the block prefix and the residual stream's tensor.

STEM = """
patches:fp32        = patchify(image) [T,PF] patch=PATCH temporal_patch=TPATCH merge=MERGE grid_h=GRID grid_w=GRID
patches.cast        = cast(patches) [T,PF] dtype=ACT
patch_embed.out.mm  = matmul(patches.cast, $w_patch_embed:w[PF,C]) [T,C]
patch_embed.out     = add(patch_embed.out.mm, $b_patch_embed:fp32[C]) [T,C]
x0                  = add(patch_embed.out, $pos_embed:fp32[T,C]) [T,C]
"""

# A pre-LayerNorm block: q/k/v projections, 2-D RoPE on q and k, attention as
# scale -> QK^T -> softmax -> PV over [H, T, D] heads, output projection and
# residual, then LayerNorm -> fc1 -> GELU(tanh) -> fc2 and residual.
BLOCK = """
{b}.ln1.out    = layernorm({x}, ${b}.ln1_w:fp32[C], ${b}.ln1_b:fp32[C]) [T,C] eps=EPS
{b}.q.out.mm   = matmul({b}.ln1.out, ${b}.wq:w[C,C]) [T,C]
{b}.q.out      = add({b}.q.out.mm, ${b}.bq:fp32[C]) [T,C]
{b}.q.h        = reshape({b}.q.out) [T,H,D] shape=(T,H,D)
{b}.q.rope     = rope_2d({b}.q.h, $rope_cos:fp32[T,D], $rope_sin:fp32[T,D]) [T,H,D]
{b}.q.t        = transpose({b}.q.rope) [H,T,D] perm=(1,0,2)
{b}.k.out.mm   = matmul({b}.ln1.out, ${b}.wk:w[C,C]) [T,C]
{b}.k.out      = add({b}.k.out.mm, ${b}.bk:fp32[C]) [T,C]
{b}.k.h        = reshape({b}.k.out) [T,H,D] shape=(T,H,D)
{b}.k.rope     = rope_2d({b}.k.h, rope_cos, rope_sin) [T,H,D]
{b}.k.t        = transpose({b}.k.rope) [H,T,D] perm=(1,0,2)
{b}.v.out.mm   = matmul({b}.ln1.out, ${b}.wv:w[C,C]) [T,C]
{b}.v.out      = add({b}.v.out.mm, ${b}.bv:fp32[C]) [T,C]
{b}.v.h        = reshape({b}.v.out) [T,H,D] shape=(T,H,D)
{b}.v.t        = transpose({b}.v.h) [H,T,D] perm=(1,0,2)
{b}.q.scaled   = scale({b}.q.t) [H,T,D] factor=QK_SCALE
{b}.k.tt       = transpose({b}.k.t) [H,D,T] perm=(0,2,1)
{b}.scores     = matmul({b}.q.scaled, {b}.k.tt) [H,T,T]
{b}.probs      = softmax({b}.scores) [H,T,T] axis=-1
{b}.ctx        = matmul({b}.probs, {b}.v.t) [H,T,D]
{b}.ctx.t      = transpose({b}.ctx) [T,H,D] perm=(1,0,2)
{b}.ctx.f      = reshape({b}.ctx.t) [T,C] shape=(T,C)
{b}.o.out.mm   = matmul({b}.ctx.f, ${b}.wo:w[C,C]) [T,C]
{b}.o.out      = add({b}.o.out.mm, ${b}.bo:fp32[C]) [T,C]
{b}.resid1     = add({x}, {b}.o.out) [T,C]
{b}.ln2.out    = layernorm({b}.resid1, ${b}.ln2_w:fp32[C], ${b}.ln2_b:fp32[C]) [T,C] eps=EPS
{b}.fc1.out.mm = matmul({b}.ln2.out, ${b}.w_fc1:w[C,FF]) [T,FF]
{b}.fc1.out    = add({b}.fc1.out.mm, ${b}.b_fc1:fp32[FF]) [T,FF]
{b}.act        = gelu_tanh({b}.fc1.out) [T,FF]
{b}.fc2.out.mm = matmul({b}.act, ${b}.w_fc2:w[FF,C]) [T,C]
{b}.fc2.out    = add({b}.fc2.out.mm, ${b}.b_fc2:fp32[C]) [T,C]
{b}.resid2     = add({b}.resid1, {b}.fc2.out) [T,C]
"""

# The patch merger: LayerNorm, each 2x2 block of tokens concatenated into one
# row (tokens are already in merge-block order), GELU(erf) MLP to the output width.
MERGER = """
merger.ln.out     = layernorm({x}, $m_ln_w:fp32[C], $m_ln_b:fp32[C]) [T,C] eps=EPS
merger.concat     = reshape(merger.ln.out) [TM,CM] shape=(TM,CM)
merger.fc1.out.mm = matmul(merger.concat, $w_m1:w[CM,CM]) [TM,CM]
merger.fc1.out    = add(merger.fc1.out.mm, $b_m1:fp32[CM]) [TM,CM]
merger.act        = gelu_erf(merger.fc1.out) [TM,CM]
merger.out.mm     = matmul(merger.act, $w_m2:w[CM,OUT]) [TM,OUT]
merger.out        = add(merger.out.mm, $b_m2:fp32[OUT]) [TM,OUT]
"""


def _symbols(cfg: VitConfig) -> dict[str, Any]:
    merged = cfg.spatial_merge_size ** 2
    return {
        "T": cfg.num_tokens, "C": cfg.hidden_size, "H": cfg.num_heads, "D": cfg.head_dim,
        "FF": cfg.intermediate_size, "OUT": cfg.out_hidden_size,
        "PF": cfg.in_channels * cfg.temporal_patch_size * cfg.patch_size ** 2,
        "TM": cfg.num_tokens // merged, "CM": cfg.hidden_size * merged,
        "PATCH": cfg.patch_size, "TPATCH": cfg.temporal_patch_size,
        "MERGE": cfg.spatial_merge_size, "GRID": cfg.grid,
        "EPS": cfg.layernorm_eps, "QK_SCALE": float(cfg.head_dim) ** -0.5,
        "ACT": cfg.act_dtype,
    }


_LINE = re.compile(r"^(?P<out>[^\s=:]+)(?::(?P<dt>\w+))?\s*=\s*(?P<kind>\w+)\((?P<args>[^)]*)\)"
                   r"\s*\[(?P<shape>[^\]]*)\]\s*(?P<attrs>.*)$")
_CONST = re.compile(r"^\$(?P<name>[^:]+):(?P<dt>\w+)\[(?P<shape>[^\]]*)\]$")


class _Program:
    """Assembles op programs into one graph: op ids in emission order."""

    def __init__(self, cfg: VitConfig) -> None:
        self.sym = _symbols(cfg)
        self.dtypes = {"w": cfg.weight_dtype, "act": cfg.act_dtype, "fp32": "fp32",
                       "fp16": "fp16", "int32": "int32"}
        self.tensors: dict[str, Tensor] = {}
        self.ops: list[Op] = []

    def _value(self, text: str) -> Any:
        text = text.strip()
        if text.startswith("("):
            return tuple(self._value(p) for p in text[1:-1].split(","))
        if text in self.sym:
            return self.sym[text]
        return ast.literal_eval(text)

    def _shape(self, text: str) -> tuple[int, ...]:
        return tuple(int(self._value(p)) for p in text.split(",")) if text.strip() else ()

    def _declare(self, t: Tensor) -> str:
        have = self.tensors.get(t.name)
        if have is not None and have != t:
            raise ValueError(f"{t.name!r} declared as {have} and as {t}")
        self.tensors[t.name] = t
        return t.name

    def _arg(self, text: str) -> str:
        m = _CONST.match(text)
        if m is None:
            if text not in self.tensors:
                raise ValueError(f"{text!r} is read before it is declared")
            return text
        return self._declare(Tensor(m["name"], self.dtypes[m["dt"]], self._shape(m["shape"]),
                                    True))

    @staticmethod
    def _split(text: str) -> list[str]:
        """Split on the commas outside [...]."""
        parts, depth, cur = [], 0, ""
        for ch in text:
            depth += (ch == "[") - (ch == "]")
            if ch == "," and depth == 0:
                parts.append(cur.strip())
                cur = ""
            else:
                cur += ch
        return parts + [cur.strip()]

    def declare_input(self, name: str, dtype: str, shape: tuple[int, ...]) -> None:
        self._declare(Tensor(name, dtype, tuple(shape)))

    def run(self, program: str, **names: str) -> None:
        for raw in program.strip().splitlines():
            line = raw.format(**names)
            m = _LINE.match(line.strip())
            if m is None:
                raise ValueError(f"cannot parse op line {line!r}")
            ins = tuple(self._arg(a) for a in self._split(m["args"]))
            out = m["out"]
            if out in self.tensors:
                raise ValueError(f"{out!r} is written twice")
            self._declare(Tensor(out, self.dtypes[m["dt"] or "act"], self._shape(m["shape"])))
            attrs = {}
            for item in m["attrs"].split():
                key, val = item.split("=", 1)
                attrs[key] = self._value(val)
            self.ops.append(Op(len(self.ops), m["kind"], ins, (out,), attrs))

    def graph(self, inputs: tuple[str, ...], outputs: tuple[str, ...]) -> Graph:
        return Graph(self.tensors, tuple(self.ops), inputs, outputs)


def build_vision_encoder(cfg: VitConfig) -> Graph:
    """The encoder graph of hexlib/models/vit.py:113-218 for `cfg`: the image
    [channels, frames, S, S] fp32 in, the merged embeddings out."""
    bad = config_problems(cfg)
    if bad:
        raise ValueError("invalid vision config: " + "; ".join(bad))
    p = _Program(cfg)
    p.declare_input("image", "fp32", (cfg.in_channels, cfg.temporal_patch_size,
                                      cfg.image_size, cfg.image_size))
    p.run(STEM)
    stream = "x0"
    for i in range(cfg.depth):
        p.run(BLOCK, b=f"blk{i}", x=stream)
        stream = f"blk{i}.resid2"
    p.run(MERGER, x=stream)
    return p.graph(("image",), ("merger.out",))


def weight_names(cfg: VitConfig) -> tuple[str, ...]:
    """Every const the encoder reads, sorted (the order feeds are drawn in)."""
    g = build_vision_encoder(cfg)
    return tuple(sorted(n for n, t in g.tensors.items() if t.const))


# ---- graph edits ----------------------------------------------------------------------

class _Edit:
    """The edits of one rewrite pass over `graph`, applied together by
    `result()`: ops replaced in place (a replacement keeps the position of the
    op it replaces), ops removed, tensors removed or added."""

    def __init__(self, graph: Graph) -> None:
        self.graph = graph
        self.readers: dict[str, list[Op]] = {}
        for op in graph.ops:
            for n in op.inputs:
                self.readers.setdefault(n, []).append(op)
        self.writer = {n: op for op in graph.ops for n in op.outputs}
        self.kept_outputs = frozenset(graph.outputs)
        self.replaced: dict[int, Op] = {}
        self.removed: set[int] = set()
        self.dead: set[str] = set()
        self.born: dict[str, Tensor] = {}

    def only_reader(self, name: str) -> Op | None:
        """The one op that reads `name`, if exactly one does and `name` is
        not a graph output (so it may disappear)."""
        r = self.readers.get(name, [])
        return r[0] if len(r) == 1 and name not in self.kept_outputs else None

    def written_by(self, name: str, kind: str) -> Op | None:
        op = self.writer.get(name)
        return op if op is not None and op.kind == kind else None

    def touched(self, op: Op) -> bool:
        return op.id in self.removed or op.id in self.replaced

    def replace(self, op: Op, new: Op) -> None:
        self.replaced[op.id] = new

    def remove(self, ops: Iterable[Op], tensors: Iterable[str] = ()) -> None:
        for op in ops:
            self.removed.add(op.id)
        self.dead.update(tensors)

    def add_tensor(self, t: Tensor) -> str:
        self.born[t.name] = t
        return t.name

    def result(self, prune_consts: bool = False) -> Graph:
        if not self.replaced and not self.removed:
            return self.graph
        ops = tuple(self.replaced.get(o.id, o) for o in self.graph.ops
                    if o.id in self.replaced or o.id not in self.removed)
        tensors = {n: t for n, t in self.graph.tensors.items() if n not in self.dead}
        tensors.update(self.born)
        if prune_consts:
            read = {n for o in ops for n in o.inputs}
            tensors = {n: t for n, t in tensors.items() if not t.const or n in read}
        return Graph(tensors, ops, self.graph.inputs, self.graph.outputs)


# ---- the reference's fusion -----------------------------------------------------------

FUSABLE_ACTS = ("gelu_tanh", "gelu_erf")


def fuse(graph: Graph) -> Graph:
    """matmul -> add of a 1-D const bias (-> GELU) becomes one
    `matmul_epilogue(a, w, bias)` with attr `act` ("none" or the GELU's kind),
    as hexlib/graph/fuse.py:16-92 folds it: the product and the biased sum
    must each be read by that next op alone and not be graph outputs; the
    fused op keeps the matmul's id and place and writes the last op's output."""
    ed = _Edit(graph)
    for mm in graph.ops:
        if mm.kind != "matmul" or ed.touched(mm):
            continue
        product = mm.outputs[0]
        add = ed.only_reader(product)
        if add is None or add.kind != "add" or len(add.inputs) != 2 or ed.touched(add):
            continue
        bias = add.inputs[1] if add.inputs[0] == product else add.inputs[0]
        bt = graph.tensors.get(bias)
        if bt is None or not bt.const or len(bt.shape) != 1:
            continue
        tail, act = add, "none"
        gelu = ed.only_reader(add.outputs[0])
        if gelu is not None and gelu.kind in FUSABLE_ACTS and not ed.touched(gelu):
            tail, act = gelu, gelu.kind
        chain = [add] if tail is add else [add, gelu]
        ed.replace(mm, Op(mm.id, "matmul_epilogue", (mm.inputs[0], mm.inputs[1], bias),
                          tail.outputs, {"act": act}))
        ed.remove(chain, [o for c in [mm] + chain[:-1] for o in c.outputs])
    return ed.result()


# ---- CUDA-only rewrites ------------------------------------------------------------------

def fuse_attention(graph: Graph) -> Graph:
    """CUDA-only: scale(q) -> matmul(., transpose_hd(k)) -> softmax -> matmul(., v)
    becomes one `attention(q, k, v)` op with attr `scale` in the place of the
    last matmul, and the [H, T, T] scores and probabilities are never
    written. Each removed intermediate must be read by the next op of the
    chain alone and not be a graph output; q, k, v and the context are fp16
    [Bn, T, D] of one shape."""
    ed = _Edit(graph)
    T = graph.tensors
    for sm in graph.ops:
        if sm.kind != "softmax" or sm.attrs.get("axis") != -1:
            continue
        qk = ed.written_by(sm.inputs[0], "matmul")
        pv = ed.only_reader(sm.outputs[0])
        if qk is None or pv is None or pv.kind != "matmul" or pv.inputs[0] != sm.outputs[0]:
            continue
        if ed.only_reader(qk.outputs[0]) is not sm:
            continue
        sc = ed.written_by(qk.inputs[0], "scale")
        kt = ed.written_by(qk.inputs[1], "transpose")
        if sc is None or kt is None or tuple(kt.attrs.get("perm", ())) != (0, 2, 1):
            continue
        if ed.only_reader(sc.outputs[0]) is not qk or ed.only_reader(kt.outputs[0]) is not qk:
            continue
        q, k, v = sc.inputs[0], kt.inputs[0], pv.inputs[1]
        shape = T[q].shape
        if len(shape) != 3 or T[k].shape != shape or T[v].shape != shape:
            continue
        if any(T[n].dtype != "fp16" for n in (q, k, v, pv.outputs[0])):
            continue
        ed.replace(pv, pv.with_(kind="attention", inputs=(q, k, v),
                                attrs={"scale": float(sc.attrs["factor"])}))
        chain = (sc, kt, qk, sm)
        ed.remove(chain, [c.outputs[0] for c in chain])
    return ed.result()


def fuse_residual(graph: Graph) -> Graph:
    """CUDA-only: `add(r, matmul_epilogue(a, w, b))` whose product nothing
    else reads becomes `matmul_epilogue_residual(a, w, b, r)` in the add's
    place (its inputs are all ready there); the epilogue rounds the product to
    fp16 before adding, as the two ops do. r must be an fp16 activation of
    the product's shape."""
    ed = _Edit(graph)
    T = graph.tensors
    for add in graph.ops:
        if add.kind != "add" or len(add.inputs) != 2 or T[add.outputs[0]].dtype != "fp16":
            continue
        for side in (1, 0):
            mm = ed.written_by(add.inputs[side], "matmul_epilogue")
            r = add.inputs[1 - side]
            if mm is None or ed.touched(mm) or ed.only_reader(mm.outputs[0]) is not add:
                continue
            rt, pt = T[r], T[mm.outputs[0]]
            if rt.const or rt.dtype != "fp16" or pt.dtype != "fp16" or rt.shape != pt.shape:
                continue
            ed.replace(add, add.with_(kind="matmul_epilogue_residual",
                                      inputs=tuple(mm.inputs) + (r,),
                                      attrs={"act": mm.attrs.get("act", "none")}))
            ed.remove([mm], mm.outputs)
            break
    return ed.result()


def fuse_patchify_cast(graph: Graph) -> Graph:
    """CUDA-only: `cast(patchify(image), fp16)` whose fp32 patch rows nothing
    else reads becomes one `patchify_cast(image)` writing the fp16 rows (each
    value rounded to nearest even, as the cast rounds it): one pass over the
    image instead of a write and a re-read of the fp32 rows."""
    ed = _Edit(graph)
    for pt in graph.ops:
        if pt.kind != "patchify":
            continue
        rows = pt.outputs[0]
        cast = ed.only_reader(rows)
        if cast is None or cast.kind != "cast" or cast.attrs.get("dtype") != "fp16":
            continue
        if graph.tensors[rows].dtype != "fp32":
            continue
        ed.replace(pt, pt.with_(kind="patchify_cast", outputs=cast.outputs))
        ed.remove([cast], [rows])
    return ed.result()


def fold_layernorm(graph: Graph, derived_in: Mapping[str, tuple] | None = None
                   ) -> tuple[Graph, dict[str, tuple]]:
    """CUDA-only, after `fuse_qkv`: a `layernorm(x, gamma, beta)` whose only
    reader is a GEMM over its output with an fp16 weight W [K, N], N a
    multiple of 256, becomes

        stats = ln_stats(x)                                   [T, 2] fp32
        out   = matmul_epilogue_ln(x, W', cols, stats)         (or ..._ln_rope)

    with W' = fp16(diag(gamma) W) and cols [2, N] = (beta @ W + b; the column
    sums of W') new consts: the GEMM's epilogue forms
    act(rstd * (x @ W' - mean * colsum) + bias) = act(LayerNorm(x) @ W + b),
    so the normalised rows are never written out and read back. The RoPE
    variant takes the two segment tables interleaved ([2T, 2, 16]). New
    consts come back as `{name: (recipe, parts, arg)}` for the batch builder."""
    ed = _Edit(graph)
    T = graph.tensors
    derived: dict[str, tuple] = {}
    for ln in graph.ops:
        if ln.kind != "layernorm" or len(ln.inputs) != 3:
            continue
        y = ln.outputs[0]
        mm = ed.only_reader(y)
        if mm is None or mm.kind not in ("matmul_epilogue", "matmul_epilogue_rope") \
                or mm.inputs[0] != y:
            continue
        x, gamma, beta = ln.inputs
        w, b = mm.inputs[1], mm.inputs[2]
        wt, bt, xt = T[w], T[b], T[x]
        consts_ok = (wt.const and wt.dtype == "fp16" and len(wt.shape) == 2 and bt.const
                     and bt.dtype == "fp32" and all(T[n].const and T[n].dtype == "fp32"
                                                    for n in (gamma, beta)))
        if not consts_ok:
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
        wf = ed.add_tensor(Tensor(f"lnfold_w({gamma},{w})", "fp16", (K, N), True))
        cols = ed.add_tensor(Tensor(f"lnfold_cols({gamma},{beta},{w},{b})", "fp32", (2, N),
                                    True))
        stats = ed.add_tensor(Tensor(f"{y}+stats", "fp32", (xt.shape[0], 2)))
        derived[wf] = ("ln_fold_w", (gamma, w), 0)
        derived[cols] = ("ln_fold_cols", (gamma, beta, w, b), 0)
        ed.replace(ln, ln.with_(kind="ln_stats", inputs=(x,), outputs=(stats,),
                                attrs={"eps": float(ln.attrs["eps"])}))
        act = {"act": mm.attrs.get("act", "none")}
        if rope_src is None:
            ed.replace(mm, mm.with_(kind="matmul_epilogue_ln", inputs=(x, wf, cols, stats),
                                    attrs=act))
        else:
            cos, sin = rope_src
            segtab = ed.add_tensor(Tensor(f"rope_segtab({cos},{sin})", "fp32",
                                          (T[mm.inputs[3]].shape[0], 2, 16), True))
            derived[segtab] = ("rope_segtab", (cos, sin), 0)
            ed.replace(mm, mm.with_(kind="matmul_epilogue_ln_rope",
                                    inputs=(x, wf, cols, stats, segtab, mm.inputs[5]),
                                    attrs=dict(act, rope_cols=int(mm.attrs["rope_cols"]))))
        ed.remove([], [y])
    if not derived:
        return graph, {}
    return ed.result(prune_consts=True), derived


def fuse_qkv(graph: Graph, rope_epilogue: bool = False) -> tuple[Graph, dict[str, tuple]]:
    """CUDA-only, after `fuse_attention`: per block, the q, k and v projections
    (three matmul_epilogue over one input), their reshapes to [T, H, D], the
    rope_2d of q and k, the three [T,H,D] -> [H,T,D] transposes into the
    attention op and the transpose of its output back to [T, H, D] become

        raw   = matmul_epilogue(a, [wq|wk|wv], [bq|bk|bv])   [T, 3, H, D]
        qkv   = rope_qk(raw, cos, sin)                       [T, 3, H, D]  (in place)
        ctx.t = attention_qkv(qkv)                           [T, H, D]

    or, with `rope_epilogue`, the rotation applied by the GEMM's epilogue
    before the one fp16 store (a q4_0 / q8_0 weight too: the session keeps an
    fp16 copy of it for the GEMM to read):

        qkv   = matmul_epilogue_rope(a, [wq|wk|wv], [bq|bk|bv],
                                     seg_cos, seg_sin, seg_idx)  [T, 3, H, D]
        ctx.t = attention_qkv(qkv)

    where seg_cos / seg_sin [2T, 16] and seg_idx [T, 2] int32 are the
    half-symmetric cos/sin tables cut into 16-wide segments and deduplicated
    (a 2-D RoPE repeats each segment across a row or column of the patch
    grid, so the distinct ones are few and stay cache-resident under the
    epilogue); the batch builder refuses tables that are not half-symmetric.

    The packed GEMM takes the q projection's place, rope_qk the k
    projection's (id and place), attention_qkv the final transpose's. The
    concatenated weight and bias and the segment tables are new consts,
    returned as `{name: ("concat", (parts...), axis)}` and
    `{name: ("rope_segments", (cos, sin), which)}` for the batch builder to
    derive from the feeds. Every removed intermediate must be read by its
    chain's next op alone and not be a graph output; anything else leaves the
    block as it was."""
    ed = _Edit(graph)
    T = graph.tensors
    derived: dict[str, tuple] = {}

    def step_back(name: str, kind: str) -> Op | None:
        """The op of `kind` that writes `name`, if `name` has one reader."""
        op = ed.written_by(name, kind)
        return op if op is not None and ed.only_reader(name) is not None else None

    def projection(name: str, roped: bool):
        """transpose <- [rope_2d <-] reshape <- matmul_epilogue (no act)."""
        tr = step_back(name, "transpose")
        if tr is None or tuple(tr.attrs.get("perm", ())) != (1, 0, 2):
            return None
        rp = step_back(tr.inputs[0], "rope_2d") if roped else None
        if roped and rp is None:
            return None
        rs = step_back((rp or tr).inputs[0], "reshape")
        mm = step_back(rs.inputs[0], "matmul_epilogue") if rs is not None else None
        if mm is None or mm.attrs.get("act", "none") != "none":
            return None
        return [o for o in (tr, rp, rs, mm) if o is not None], mm, rp

    for att in graph.ops:
        if att.kind != "attention":
            continue
        found = [projection(n, roped) for n, roped in zip(att.inputs, (True, True, False))]
        if any(f is None for f in found):
            continue
        back = ed.only_reader(att.outputs[0])
        if back is None or back.kind != "transpose" or \
                tuple(back.attrs.get("perm", ())) != (1, 0, 2):
            continue
        mms = [f[1] for f in found]
        a = mms[0].inputs[0]
        rq, rk = found[0][2], found[1][2]
        if any(m.inputs[0] != a for m in mms) or rq.inputs[1:] != rk.inputs[1:]:
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
        heads, n_tok, d = T[att.outputs[0]].shape
        K = T[ws[0]].shape[0]
        if any(T[w].shape != (K, heads * d) for w in ws) or T[a].shape != (n_tok, K) or d != 64:
            continue
        width = 3 * heads * d
        wname = ed.add_tensor(Tensor(f"concat({ws[0]},{ws[1]},{ws[2]})", wdt, (K, width), True))
        bname = ed.add_tensor(Tensor(f"concat({bs[0]},{bs[1]},{bs[2]})", "fp32", (width,), True))
        derived[wname] = ("concat", tuple(ws), 1)
        derived[bname] = ("concat", tuple(bs), 0)
        qkv = ed.add_tensor(Tensor(f"{mms[0].outputs[0]}+qkv", "fp16", (n_tok, 3, heads, d)))
        for f in found:
            ed.remove(f[0], [o.outputs[0] for o in f[0]])
        ed.remove([att], att.outputs)
        if rope_epilogue:
            segs = []
            for i, (part, dt, shape) in enumerate((("cos", "fp32", (2 * n_tok, 16)),
                                                   ("sin", "fp32", (2 * n_tok, 16)),
                                                   ("idx", "int32", (n_tok, 2)))):
                sname = ed.add_tensor(Tensor(f"rope_segments({cos},{sin}).{part}", dt, shape,
                                             True))
                derived[sname] = ("rope_segments", (cos, sin), i)
                segs.append(sname)
            ed.replace(mms[0], Op(mms[0].id, "matmul_epilogue_rope",
                                  (a, wname, bname, *segs), (qkv,),
                                  {"act": "none", "rope_cols": 2 * heads * d}))
        else:
            raw = ed.add_tensor(Tensor(f"{mms[0].outputs[0]}+qkv.raw", "fp16",
                                       (n_tok, 3, heads, d)))
            ed.replace(mms[0], Op(mms[0].id, "matmul_epilogue", (a, wname, bname), (raw,),
                                  {"act": "none"}))
            ed.replace(mms[1], Op(mms[1].id, "rope_qk", (raw, cos, sin), (qkv,), {}))
        ed.replace(back, back.with_(kind="attention_qkv", inputs=(qkv,),
                                    attrs={"scale": float(att.attrs["scale"])}))
    if not derived:
        return graph, {}
    return ed.result(prune_consts=True), derived


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
