"""A whole compiled plan -> ONE batch blob for the CUDA dispatcher, over two
device buffers: the shared consts and a per-image region.

The CUDA analogue of hexlib/exec/wholeplan.py:92-357 (`build_whole_plan_batch`):
the same walk over the plan's steps, the same variant selection per op
(`runner.select`), reshapes emitted as no op but as a second tensor descriptor
on the same bytes, and the same blob format (`wire.pack_batch`). What differs
is the arena, because the GPU runs B images per launch:

  buffer 0 (fd CONST_FD)   every const, each at its own 256-byte-aligned
                           offset, staged once per session in the dtype its
                           consuming kernel takes.
  buffer 1 (fd IMAGE_FD)   every activation and every graph input/output, at
                           PER-IMAGE offsets, flagged BUF_PER_IMAGE: with B
                           images the dispatcher gives each tensor B
                           contiguous copies, so each kernel sees [B, ...].

`alias=True` lets activations whose lifetimes do not overlap share bytes, with
liveness computed on the plan's own op order and every reshape chain unified
into its storage owner first -- the "reshape unification" that the reference's
builder refuses without (wholeplan.py:235-258, 360-409). Graph inputs and
outputs are never aliased.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Mapping

import numpy as np

from hexlib_b200 import runner, wire
from hexlib_b200 import quant
from hexlib_b200.graph import as_graph, nbytes as ir_nbytes

CONST_FD = 0
IMAGE_FD = 1
ALIGN = 256

_NP = {"fp32": np.float32, "fp16": np.float16, "int32": np.int32}

# kinds whose output may share its first input's storage: their kernels read
# each element before writing it, and the rewrite that emits them leaves the
# input with no other consumer (checked below)
INPLACE_KINDS = frozenset({"rope_qk"})


class WholePlanError(Exception):
    pass


def _align(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def _ne(shape) -> tuple[int, int, int, int]:
    if len(shape) > 4:
        raise WholePlanError(f"shape {tuple(shape)} has more than 4 dims; ne is fixed at 4")
    return tuple(int(s) for s in shape) + (1,) * (4 - len(shape))


@dataclass(frozen=True)
class Placement:
    name: str
    buffer: int          # CONST_FD or IMAGE_FD
    offset: int          # per-image offset for IMAGE_FD tensors
    nbytes: int          # per image
    dtype: str
    shape: tuple[int, ...]
    region: str          # "const" | "act" | "io" | "reshape-alias"


@dataclass
class CudaPlan:
    blob: bytes
    const_payload: bytearray | None
    const_bytes: int
    image_bytes: int                     # per-image region size
    placements: dict[str, Placement]
    index: dict[str, int]                # tensor name -> wire tensor index
    n_ops: int
    op_names: tuple[str, ...]
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]
    skipped_reshapes: int
    kinds: tuple[str, ...] = field(default=())

    def response_capacity(self) -> int:
        return wire.response_capacity(self.n_ops)


def _steps(compiled):
    for s in compiled.plan.steps:
        op = getattr(s, "op", None)
        if op is not None:
            yield op


def _allocate_aliased(names, first, last, size) -> tuple[dict[str, int], int]:
    """First-fit by decreasing size over [first, last] op-index lifetimes."""
    placed: list[tuple[int, int, int, int]] = []  # (offset, end, first, last)
    offs: dict[str, int] = {}
    for n in sorted(names, key=lambda k: (-size[k], k)):
        lo, hi, sz = first[n], last[n], size[n]
        clashes = sorted((o, e) for (o, e, f, l) in placed if f <= hi and lo <= l)
        cand = 0
        for o, e in clashes:
            if cand + sz <= o:
                break
            cand = max(cand, _align(e))
        offs[n] = cand
        placed.append((cand, cand + sz, lo, hi))
    end = max((o + size[n] for n, o in offs.items()), default=0)
    return offs, _align(end)


def _is_raw(v) -> bool:
    """Packed block-quantized bytes rather than a dense value."""
    return isinstance(v, (bytes, bytearray)) or (isinstance(v, np.ndarray) and v.dtype == np.uint8)


def _concat_raw(parts, dtype: str, shape, axis: int) -> bytes:
    """Concatenate packed [K, N_i] weights along N: row by row, since each row
    of a block-quantized matrix is its own run of blocks."""
    if axis not in (1, -1) or len(shape) != 2:
        raise WholePlanError("packed weights concatenate only along the last axis of a matrix")
    K = shape[0]
    rows = [np.frombuffer(bytes(np.asarray(q, np.uint8).tobytes()) if not isinstance(q, bytes)
                          else q, np.uint8).reshape(K, -1) for q in parts]
    return np.concatenate(rows, axis=1).tobytes()


def rope_segments(cos, sin) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Cut half-symmetric [T, 64] cos/sin tables (dims i and i + 32 equal, as
    a rotate-half table built from one frequency list is) into 16-wide
    segments of dims 0..31 and keep each distinct (cos, sin) segment once:
    `(seg_cos [2T, 16], seg_sin [2T, 16], seg_idx [T, 2] int32)`, with dims
    [16s, 16s + 16) and [32 + 16s, 48 + 16s) of token t in row seg_idx[t, s]
    of both tables (rows past the distinct ones are zero). Segments are
    compared on their fp32 bits, so every value the GEMM epilogue reads is
    the table's own. Tables that are not half-symmetric are refused: the
    rotation then runs as its own op."""
    c = np.ascontiguousarray(np.asarray(cos, np.float32))
    s = np.ascontiguousarray(np.asarray(sin, np.float32))
    if c.ndim != 2 or c.shape != s.shape or c.shape[1] != 64:
        raise WholePlanError(f"rope tables must be two [T, 64] arrays; got {c.shape}, {s.shape}")
    cu, su = c.view(np.uint32), s.view(np.uint32)
    if not (np.array_equal(cu[:, :32], cu[:, 32:]) and np.array_equal(su[:, :32], su[:, 32:])):
        raise WholePlanError("the RoPE epilogue needs half-symmetric cos/sin tables "
                             "(dims i and i + 32 equal); compile without rope_epilogue")
    T = c.shape[0]
    keys = np.concatenate([cu[:, :32].reshape(2 * T, 16), su[:, :32].reshape(2 * T, 16)], axis=1)
    uniq, inverse = np.unique(keys, axis=0, return_inverse=True)
    n = uniq.shape[0]
    seg_cos = np.zeros((2 * T, 16), np.float32)
    seg_sin = np.zeros((2 * T, 16), np.float32)
    seg_cos[:n] = uniq[:, :16].view(np.float32)
    seg_sin[:n] = uniq[:, 16:].view(np.float32)
    return seg_cos, seg_sin, inverse.reshape(T, 2).astype(np.int32)


def _fp16_exact(v) -> np.ndarray:
    """A weight as the fp16 tensor the plan would stage, in float64."""
    return np.asarray(v, np.float32).astype(np.float16).astype(np.float64)


def ln_fold_w(gamma, w) -> np.ndarray:
    """diag(gamma) W rounded once to fp16: the weight a layernorm-folded GEMM
    multiplies the raw rows by."""
    return (np.asarray(gamma, np.float64)[:, None] * _fp16_exact(w)).astype(np.float16)


def ln_fold_cols(gamma, beta, w, b) -> np.ndarray:
    """[2, N] fp32: (beta @ W + b; the column sums of ln_fold_w(gamma, W)),
    both summed in float64 and rounded once."""
    wf = ln_fold_w(gamma, w).astype(np.float64)
    bias = np.asarray(beta, np.float64) @ _fp16_exact(w) + np.asarray(b, np.float64)
    return np.stack([bias, wf.sum(axis=0)]).astype(np.float32)


class _Deriver:
    """The value of a const: a feed, or built by its recipe from feeds and
    other derived consts (each built once)."""

    def __init__(self, derived, feeds, placements):
        self.derived, self.feeds, self.placements = derived, feeds, placements
        self.memo: dict[str, Any] = {}
        self.segments: dict[tuple, tuple] = {}

    def __call__(self, n: str):
        if n in self.memo:
            return self.memo[n]
        if n in self.derived:
            v = self._build(n, *self.derived[n])
        elif n in self.feeds:
            v = self.feeds[n]
        else:
            raise WholePlanError(f"no feed supplied for const {n!r}")
        self.memo[n] = v
        return v

    def _build(self, n, how, parts, arg):
        if how not in ("concat", "rope_segments", "rope_segtab", "ln_fold_w", "ln_fold_cols"):
            raise WholePlanError(f"const {n!r}: unknown derivation {how!r}")
        missing = [q for q in parts if q not in self.feeds and q not in self.derived]
        if missing:
            raise WholePlanError(f"const {n!r} is built from {missing}, not supplied")
        vals = [self(q) for q in parts]
        if how in ("rope_segments", "rope_segtab"):
            key = tuple(parts)
            if key not in self.segments:
                self.segments[key] = rope_segments(vals[0], vals[1])
            seg_cos, seg_sin, idx = self.segments[key]
            if how == "rope_segtab":
                return np.stack([seg_cos, seg_sin], axis=1)
            return (seg_cos, seg_sin, idx)[arg]
        if how == "ln_fold_w":
            return ln_fold_w(*vals)
        if how == "ln_fold_cols":
            return ln_fold_cols(*vals)
        p = self.placements.get(n)
        if p is not None and p.dtype in quant.BLOCK_BYTES and any(_is_raw(v) for v in vals):
            return _concat_raw(vals, p.dtype, p.shape, arg)
        return np.concatenate([np.asarray(v) for v in vals], axis=arg)


def build_cuda_plan(compiled, feeds: Mapping[str, Any] | None = None,
                    alias: bool = False) -> CudaPlan:
    """Pack `compiled`'s whole plan into one blob; stage `feeds`' consts if
    given. `compiled` is anything with `.graph` and `.plan.steps[i].op`: the
    reference's `Compiled` or this package's `ExecPlan`."""
    graph = as_graph(compiled.graph)
    tensors = graph.tensors
    order = list(_steps(compiled))
    if not order:
        raise WholePlanError("the plan has no ops")
    io_names = set(graph.inputs) | set(graph.outputs)
    const_names = {n for n, t in tensors.items() if t.const}

    # Outputs stored on their input's bytes: reshape (a reinterpretation) and
    # the in-place kinds, whose kernels read every element before writing it.
    reshape_src: dict[str, str] = {}
    for op in order:
        if op.kind == "reshape" or op.kind in INPLACE_KINDS:
            reshape_src[op.outputs[0]] = op.inputs[0]

    for i, op in enumerate(order):
        if op.kind in INPLACE_KINDS:
            src = op.inputs[0]
            later = [o.id for o in order[i + 1:] if src in o.inputs]
            if later or src in io_names:
                raise WholePlanError(
                    f"op {op.id} ({op.kind}) would overwrite {src!r}, which ops {later} "
                    "still read (or the host reads); it cannot run in place")

    def owner(name: str) -> str:
        seen = {name}
        while name in reshape_src:
            name = reshape_src[name]
            if name in seen:
                raise WholePlanError(f"reshape chain cycles at {name!r}")
            seen.add(name)
        return name

    aliased_io = sorted(n for n in reshape_src if n in io_names)
    if aliased_io:
        raise WholePlanError(f"graph inputs/outputs {aliased_io} are reshape outputs; "
                             "give them their own storage first")

    # ---- select every op's variant and claim dtypes -------------------------
    specs: dict[int, tuple[str, runner.CudaSpec]] = {}
    for op in order:
        if op.kind == "reshape":
            continue
        dts = tuple(tensors[n].dtype for n in op.inputs)
        try:
            name, spec = runner.select(op.kind, dict(op.attrs), dts)
            spec.check_requires(dict(op.attrs))
        except (KeyError, ValueError) as e:
            raise WholePlanError(f"op {op.id} ({op.kind}): {e}") from e
        for n in op.outputs:
            if spec.out_dtype != "any" and tensors[n].dtype != spec.out_dtype:
                raise WholePlanError(
                    f"op {op.id} ({op.kind}) writes {n!r} as {tensors[n].dtype}; "
                    f"the kernel writes {spec.out_dtype}")
        specs[op.id] = (name, spec)

    def tbytes(n: str) -> int:
        return ir_nbytes(tensors[n].shape, tensors[n].dtype)

    placements: dict[str, Placement] = {}

    # ---- consts --------------------------------------------------------------
    cursor = 0
    used = {n for op in order for n in op.inputs}
    for n in sorted(const_names):
        if n not in used:
            continue
        t = tensors[n]
        placements[n] = Placement(n, CONST_FD, cursor, tbytes(n), t.dtype, t.shape, "const")
        cursor = _align(cursor + tbytes(n))
    const_bytes = max(cursor, ALIGN)

    # ---- per-image region ------------------------------------------------------
    act_names = sorted({n for op in order for n in tuple(op.inputs) + tuple(op.outputs)
                        if n not in const_names and n not in io_names
                        and n not in reshape_src})
    cursor = 0
    io_sorted = sorted(io_names)
    for n in io_sorted:
        t = tensors[n]
        placements[n] = Placement(n, IMAGE_FD, cursor, tbytes(n), t.dtype, t.shape, "io")
        cursor = _align(cursor + tbytes(n))
    io_end = cursor
    if alias:
        first: dict[str, int] = {}
        last: dict[str, int] = {}
        for i, op in enumerate(order):
            for n in op.outputs:
                o = owner(n)
                first.setdefault(o, i)
                last[o] = max(last.get(o, i), i)
            for n in op.inputs:
                o = owner(n)
                if o in first:
                    last[o] = max(last[o], i)
        missing = [n for n in act_names if n not in first]
        if missing:
            raise WholePlanError(f"activations read but never written: {missing[:5]}")
        size = {n: tbytes(n) for n in act_names}
        offs, span = _allocate_aliased(act_names, first, last, size)
        for n in act_names:
            t = tensors[n]
            placements[n] = Placement(n, IMAGE_FD, io_end + offs[n], size[n], t.dtype,
                                      t.shape, "act")
        cursor = io_end + span
    else:
        for n in act_names:
            t = tensors[n]
            placements[n] = Placement(n, IMAGE_FD, cursor, tbytes(n), t.dtype, t.shape, "act")
            cursor = _align(cursor + tbytes(n))
    image_bytes = max(cursor, ALIGN)

    for n in reshape_src:
        o = owner(n)
        if o not in placements:
            raise WholePlanError(f"reshape {n!r} resolves to unplaced {o!r}")
        base = placements[o]
        if tbytes(n) != base.nbytes:
            raise WholePlanError(f"reshape {n!r} changes the byte count")
        t = tensors[n]
        placements[n] = Placement(n, base.buffer, base.offset, base.nbytes, t.dtype, t.shape,
                                  "reshape-alias")

    # ---- stage consts --------------------------------------------------------------
    payload = None
    derived = dict(getattr(compiled, "derived", {}) or {})
    if feeds is not None:
        payload = bytearray(const_bytes)
        resolve = _Deriver(derived, feeds, placements)
        for n, p in placements.items():
            if p.region != "const":
                continue
            value = resolve(n)
            if p.dtype in quant.BLOCK_BYTES:
                # a dense weight is quantized here, as the reference's batch
                # builder does (wholeplan.py:293-307); packed bytes pass as is
                raw = (bytes(np.asarray(value, np.uint8).tobytes()) if _is_raw(value)
                       else quant.quantize(np.asarray(value, np.float32), p.dtype))
                if len(raw) != p.nbytes:
                    raise WholePlanError(f"const {n!r}: {len(raw)} {p.dtype} bytes, "
                                         f"declared {p.nbytes}")
                payload[p.offset:p.offset + len(raw)] = raw
                continue
            a = np.ascontiguousarray(np.asarray(value), dtype=_NP[p.dtype])
            if tuple(a.shape) != tuple(p.shape):
                raise WholePlanError(f"feed {n!r} has shape {a.shape}, declared {p.shape}")
            raw = a.tobytes()
            payload[p.offset:p.offset + len(raw)] = raw

    # ---- wire descriptors ----------------------------------------------------------
    names = sorted(placements)
    index = {n: i for i, n in enumerate(names)}
    wt = [wire.TensorDesc(bi=0 if placements[n].buffer == CONST_FD else 1,
                          offset=placements[n].offset, nbytes=placements[n].nbytes,
                          dtype=placements[n].dtype, layout="row_major",
                          ne=_ne(placements[n].shape)) for n in names]
    ops: list[wire.OpDesc] = []
    op_names: list[str] = []
    kinds: list[str] = []
    skipped = 0
    for op in order:
        if op.kind == "reshape":
            skipped += 1
            continue
        vname, spec = specs[op.id]
        ops.append(wire.OpDesc(kind=runner.KIND_ID[vname],
                               params=runner.encode_params(spec, dict(op.attrs)),
                               src=tuple(index[n] for n in op.inputs),
                               dst=tuple(index[n] for n in op.outputs)))
        op_names.append(f"{op.id}:{vname}")
        kinds.append(vname)
    bufs = [wire.BufDesc(fd=CONST_FD, size=const_bytes, flags=0),
            wire.BufDesc(fd=IMAGE_FD, size=image_bytes, flags=wire.BUF_PER_IMAGE)]
    blob = wire.pack_batch(bufs, wt, ops)
    return CudaPlan(blob=blob, const_payload=payload, const_bytes=const_bytes,
                    image_bytes=image_bytes, placements=placements, index=index,
                    n_ops=len(ops), op_names=tuple(op_names), inputs=tuple(graph.inputs),
                    outputs=tuple(graph.outputs), skipped_reshapes=skipped,
                    kinds=tuple(kinds))
