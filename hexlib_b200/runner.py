"""Kernel variants of the CUDA backend and the selection of one per op.

Mirrors hexlib/exec/runner.py:379-702 (`RunnerSpec`, `SPECS`, `select`) and
hexlib/runtime/genentry.py:67-88 (`KIND_ID`) for the wire path: one spec per
KERNEL VARIANT, selected from the op kind and its attrs (and, here, the input
dtypes), refusing -- never defaulting -- when no variant or more than one
accepts. The wire carries no attrs, so `select` is where `perm` and `axis`
decide the variant, and `encode_params` is where attr-sourced scalars become
the op's int32 params (floats as their IEEE-754 bits, dsp.py:286-305).

DIFFERENCES FROM THE DSP's TABLE, each deliberate:
  * matmul_epilogue takes an fp16 [K, N] weight as well as the DSP's q4_0
    one (and q8_0): a block-quantized weight is dequantized to fp16 -- every
    value rounded as the DSP kernel rounds it -- ahead of the tensor-core
    GEMM, in a scratch the session owns.
  * add's right operand may be fp32: the pos_embed add then rounds once,
    exactly as the numpy executor computes it, instead of pre-rounding the
    table to fp16 as the DSP spec does (runner.py:395-398).
  * reshape has a variant (a device copy): the batch builder still elides
    reshapes by aliasing, but a blob that carries one is served.
  * ids are appended for kernels the DSP table does not have: attention (13),
    rmsnorm (14), matmul_epilogue_residual (15), matmul_epilogue_rope (16),
    attention_qkv (17), rope_qk (18), ln_stats (19), matmul_epilogue_ln (20),
    matmul_epilogue_ln_rope (21) and patchify_cast (22).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Any, Mapping

KIND_ID: dict[str, int] = {
    "add": 1,
    "cast": 2,
    "layernorm": 3,
    "matmul": 4,
    "matmul_epilogue": 5,
    "patchify": 6,
    "reshape": 7,
    "rope_2d": 8,
    "scale": 9,
    "softmax": 10,
    "transpose": 11,
    "transpose_hd": 12,
    # appended: kernels the DSP table does not have
    "attention": 13,
    "rmsnorm": 14,
    "matmul_epilogue_residual": 15,
    "matmul_epilogue_rope": 16,
    "attention_qkv": 17,
    "rope_qk": 18,
    "ln_stats": 19,
    "matmul_epilogue_ln": 20,
    "matmul_epilogue_ln_rope": 21,
    "patchify_cast": 22,
}

ACT_CODES = (("none", 0), ("gelu_tanh", 1), ("gelu_erf", 2))


@dataclass(frozen=True)
class Param:
    """One attr-sourced scalar carried in the op's params, in order."""
    attr: str
    ctype: str = "int"            # "int" | "float"
    codes: tuple[tuple[str, int], ...] = ()

    def encode(self, attrs: Mapping[str, Any]) -> int:
        if self.attr not in attrs:
            raise KeyError(f"param wants attr {self.attr!r}; op attrs are {sorted(attrs)}")
        v = attrs[self.attr]
        if self.codes:
            table = dict(self.codes)
            if v not in table:
                raise ValueError(f"{self.attr}={v!r} is not one of {sorted(table)}; "
                                 "refused rather than defaulted")
            return table[v]
        if self.ctype == "int":
            return int(v)
        return struct.unpack("<i", struct.pack("<f", float(v)))[0]


@dataclass(frozen=True)
class CudaSpec:
    kind: str                                 # op kind this variant implements
    inputs: tuple[tuple[str, ...], ...]       # accepted dtypes per input
    out_dtype: str
    params: tuple[Param, ...] = ()
    requires: tuple[tuple[str, Any], ...] = ()
    entry: str = ""                           # the C-ABI per-kernel entry

    def accepts(self, attrs: Mapping[str, Any]) -> bool:
        return all(_norm(attrs.get(k)) == _norm(v) for k, v in self.requires)

    def check_requires(self, attrs: Mapping[str, Any]) -> None:
        for k, want in self.requires:
            if _norm(attrs.get(k)) != _norm(want):
                raise ValueError(
                    f"this kernel implements {self.kind} only for {k}={want!r}, "
                    f"not {attrs.get(k)!r}; dispatching it would give a "
                    "correctly-shaped wrong answer")

    def check_dtypes(self, dtypes: tuple[str, ...]) -> None:
        if len(dtypes) != len(self.inputs):
            raise ValueError(f"{self.kind} takes {len(self.inputs)} inputs, got {len(dtypes)}")
        for i, (d, ok) in enumerate(zip(dtypes, self.inputs)):
            if d not in ok:
                raise ValueError(f"{self.kind} input {i} is {d!r}; this kernel takes {ok}")

    def buf_layouts(self) -> tuple[str, ...]:
        return ("row_major",) * (len(self.inputs) + 1)


def _norm(v):
    if isinstance(v, list):
        return tuple(v)
    return v


F16, F32 = ("fp16",), ("fp32",)
# a matmul weight: fp16, or block-quantized (dequantized to fp16 ahead of the GEMM)
WEIGHT = ("fp16", "q4_0", "q8_0")

SPECS: dict[str, CudaSpec] = {
    "add": CudaSpec("add", (F16, ("fp16", "fp32")), "fp16", entry="hexlib_b200_add_fp16"),
    "cast": CudaSpec("cast", (F32,), "fp16", requires=(("dtype", "fp16"),),
                     entry="hexlib_b200_cast_f32_f16"),
    "layernorm": CudaSpec("layernorm", (F16, F32, F32), "fp16",
                          params=(Param("eps", "float"),), entry="hexlib_b200_layernorm_fp16"),
    "matmul": CudaSpec("matmul", (F16, F16), "fp16", entry="hexlib_b200_matmul_fp16"),
    "matmul_epilogue": CudaSpec("matmul_epilogue", (F16, WEIGHT, F32), "fp16",
                                params=(Param("act", "int", ACT_CODES),),
                                entry="hexlib_b200_matmul_epilogue_fp16"),
    "patchify": CudaSpec("patchify", (F32,), "fp32",
                         params=(Param("patch"), Param("merge"), Param("grid_h"),
                                 Param("grid_w")),
                         entry="hexlib_b200_patchify_fp32"),
    "reshape": CudaSpec("reshape", (("fp16", "fp32", "int32"),), "any"),
    "rope_2d": CudaSpec("rope_2d", (F16, F32, F32), "fp16", entry="hexlib_b200_rope_2d_fp16"),
    "scale": CudaSpec("scale", (F16,), "fp16", params=(Param("factor", "float"),),
                      entry="hexlib_b200_scale_fp16"),
    "softmax": CudaSpec("softmax", (F16,), "fp16", requires=(("axis", -1),),
                        entry="hexlib_b200_softmax_fp16"),
    "transpose": CudaSpec("transpose", (F16,), "fp16", requires=(("perm", (1, 0, 2)),),
                          entry="hexlib_b200_transpose_th_fp16"),
    "transpose_hd": CudaSpec("transpose", (F16,), "fp16", requires=(("perm", (0, 2, 1)),),
                             entry="hexlib_b200_transpose_hd_fp16"),
    "attention": CudaSpec("attention", (F16, F16, F16), "fp16",
                          params=(Param("scale", "float"),), entry="hexlib_b200_attention_fp16"),
    "rmsnorm": CudaSpec("rmsnorm", (F16, F16), "fp16", params=(Param("eps", "float"),),
                        entry="hexlib_b200_rmsnorm_fp16"),
    "matmul_epilogue_residual": CudaSpec(
        "matmul_epilogue_residual", (F16, WEIGHT, F32, F16), "fp16",
        params=(Param("act", "int", ACT_CODES),),
        entry="hexlib_b200_matmul_epilogue_residual_fp16"),
    "matmul_epilogue_rope": CudaSpec(
        "matmul_epilogue_rope", (F16, WEIGHT, F32, F32, F32, ("int32",)), "fp16",
        params=(Param("act", "int", ACT_CODES), Param("rope_cols")),
        entry="hexlib_b200_matmul_epilogue_rope_fp16"),
    "rope_qk": CudaSpec("rope_qk", (F16, F32, F32), "fp16", entry="hexlib_b200_rope_qk_fp16"),
    "patchify_cast": CudaSpec("patchify_cast", (F32,), "fp16",
                              params=(Param("patch"), Param("merge"), Param("grid_h"),
                                      Param("grid_w")),
                              entry="hexlib_b200_patchify_fp16"),
    "ln_stats": CudaSpec("ln_stats", (F16,), "fp32", params=(Param("eps", "float"),),
                         entry="hexlib_b200_ln_stats_fp16"),
    "matmul_epilogue_ln": CudaSpec(
        "matmul_epilogue_ln", (F16, F16, F32, F32), "fp16",
        params=(Param("act", "int", ACT_CODES),),
        entry="hexlib_b200_matmul_epilogue_ln_fp16"),
    "matmul_epilogue_ln_rope": CudaSpec(
        "matmul_epilogue_ln_rope", (F16, F16, F32, F32, F32, ("int32",)), "fp16",
        params=(Param("act", "int", ACT_CODES), Param("rope_cols")),
        entry="hexlib_b200_matmul_epilogue_ln_rope_fp16"),
    "attention_qkv": CudaSpec("attention_qkv", (F16,), "fp16",
                              params=(Param("scale", "float"),),
                              entry="hexlib_b200_attention_qkv_fp16"),
}


def variants_for(kind: str) -> tuple[str, ...]:
    return tuple(n for n, s in SPECS.items() if s.kind == kind)


def select(kind: str, attrs: Mapping[str, Any],
           dtypes: tuple[str, ...] | None = None) -> tuple[str, CudaSpec]:
    """The one variant of `kind` that accepts these attrs (and input dtypes):
    `(variant_name, spec)`. No candidate, or several, is an error
    (runner.py:641-687)."""
    cands = [(n, s) for n, s in SPECS.items() if s.kind == kind]
    if not cands:
        raise KeyError(f"no CUDA kernel implements {kind!r}; known kinds are "
                       f"{sorted({s.kind for s in SPECS.values()})}")
    ok = [(n, s) for n, s in cands if s.accepts(attrs)]
    if len(ok) > 1:
        raise ValueError(f"{len(ok)} {kind!r} kernels accept this op "
                         f"({[n for n, _ in ok]}); their requires are not disjoint")
    if not ok:
        detail = "; ".join(f"{n} requires {dict(s.requires)}" for n, s in cands)
        raise ValueError(f"no {kind!r} kernel accepts attrs {dict(attrs)}: {detail}")
    name, spec = ok[0]
    if dtypes is not None:
        spec.check_dtypes(tuple(dtypes))
    return name, spec


def encode_params(spec: CudaSpec, attrs: Mapping[str, Any]) -> tuple[int, ...]:
    return tuple(p.encode(attrs) for p in spec.params)
