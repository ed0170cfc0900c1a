"""Upstream (transformers Qwen3.5 vision tower) parameters -> the encoder
graph's const feeds: the counterpart of hexlib/models/loader.py:149-227
`feeds_from_params`, so a real checkpoint (or the reference's tiny golden)
feeds the CUDA plan exactly as it feeds the reference's executor.

The mapping is a table: each graph const names the upstream parameter it
comes from and one reshaping rule --

  linear    an nn.Linear weight, stored [out, in], used as [in, out]
  as_is     a bias or a LayerNorm weight/shift, copied
  qkv i     block i (0 q, 1 k, 2 v) of the fused [3C, C] qkv projection's
            rows -- the attention forward unbinds its output along a leading
            axis of 3 -- then, for the weight, [out, in] -> [in, out]
  conv      the Conv3d patch embedding [E, C, T, p, p], flattened over
            (C, T, p, p) -- patchify's feature order -- and used as [feat, E]

Three consts are not read but derived, as upstream derives them at run time
for the configured resolution:

  pos_embed        the learned `side x side` grid of position embeddings
                   bilinearly resampled onto this patch grid (sample points
                   evenly spaced over [0, side - 1] along each axis, the four
                   neighbouring grid rows weighted by the fractional
                   distances, accumulated in float64), in merge-block token
                   order; `side` is the square root of the table's rows.
  rope_cos/sin     the 2-D rotary tables (feeds.rope_tables).

Every feed is checked against the graph's declared shape: at width 768 each
projection is square, so a missing transpose would pass a shape check only
by luck of a non-square one -- the test pins the values, not the shapes.
"""
from __future__ import annotations

import math
from typing import Callable

import numpy as np

from hexlib_b200.feeds import rope_tables, vision_position_ids
from hexlib_b200.graph import Graph, VitConfig


def _rules(cfg: VitConfig) -> dict[str, tuple]:
    """graph const -> (upstream parameter, rule, rule argument)."""
    table = {
        "w_patch_embed": ("patch_embed.proj.weight", "conv", None),
        "b_patch_embed": ("patch_embed.proj.bias", "as_is", None),
        "m_ln_w": ("merger.norm.weight", "as_is", None),
        "m_ln_b": ("merger.norm.bias", "as_is", None),
        "w_m1": ("merger.linear_fc1.weight", "linear", None),
        "b_m1": ("merger.linear_fc1.bias", "as_is", None),
        "w_m2": ("merger.linear_fc2.weight", "linear", None),
        "b_m2": ("merger.linear_fc2.bias", "as_is", None),
    }
    for i in range(cfg.depth):
        up, me = f"blocks.{i}", f"blk{i}"
        for j, which in enumerate("qkv"):
            table[f"{me}.w{which}"] = (f"{up}.attn.qkv.weight", "qkv", j)
            table[f"{me}.b{which}"] = (f"{up}.attn.qkv.bias", "qkv", j)
        table[f"{me}.wo"] = (f"{up}.attn.proj.weight", "linear", None)
        table[f"{me}.bo"] = (f"{up}.attn.proj.bias", "as_is", None)
        table[f"{me}.w_fc1"] = (f"{up}.mlp.linear_fc1.weight", "linear", None)
        table[f"{me}.b_fc1"] = (f"{up}.mlp.linear_fc1.bias", "as_is", None)
        table[f"{me}.w_fc2"] = (f"{up}.mlp.linear_fc2.weight", "linear", None)
        table[f"{me}.b_fc2"] = (f"{up}.mlp.linear_fc2.bias", "as_is", None)
        for n in ("1", "2"):
            table[f"{me}.ln{n}_w"] = (f"{up}.norm{n}.weight", "as_is", None)
            table[f"{me}.ln{n}_b"] = (f"{up}.norm{n}.bias", "as_is", None)
    return table


def _apply(rule: str, arg, x: np.ndarray, width: int) -> np.ndarray:
    if rule == "as_is":
        return x
    if rule == "linear":
        return x.T
    if rule == "conv":
        return x.reshape(x.shape[0], -1).T
    if rule == "qkv":
        part = x[arg * width:(arg + 1) * width]
        return part.T if part.ndim == 2 else part
    raise ValueError(f"unknown rule {rule!r}")


def resample_pos_embed(table: np.ndarray, grid: int, merge: int) -> np.ndarray:
    """The learned [side^2, C] position grid bilinearly resampled to this
    [grid^2, C] patch grid in merge-block token order (float32)."""
    side = math.isqrt(table.shape[0])
    if side * side != table.shape[0]:
        raise ValueError(f"pos_embed has {table.shape[0]} rows: not a square grid")
    at = np.linspace(0, side - 1, grid)
    lo = at.astype(np.int64)
    hi = np.minimum(lo + 1, side - 1)
    frac = at - lo
    rows, cols = vision_position_ids(grid, merge).T          # token -> (row, col)
    src = table.astype(np.float64)
    out = np.zeros((rows.size, table.shape[1]), np.float64)
    for r_idx, r_w in ((lo, 1.0 - frac), (hi, frac)):
        for c_idx, c_w in ((lo, 1.0 - frac), (hi, frac)):
            weight = r_w[rows] * c_w[cols]
            out += src[r_idx[rows] * side + c_idx[cols]] * weight[:, None]
    return out.astype(np.float32)


def feeds_from_params(graph: Graph, cfg: VitConfig,
                      get: Callable[[str], np.ndarray]) -> dict[str, np.ndarray]:
    """A feed for every const of `graph` (the encoder of `cfg`) from the
    upstream parameters, `get(name)` returning each as an array. Raises
    ValueError on a const the mapping does not cover, a feed for a tensor the
    graph does not declare as const, or a shape the graph does not declare."""
    feeds = {name: _apply(rule, arg, np.asarray(get(src)), cfg.hidden_size)
             for name, (src, rule, arg) in _rules(cfg).items()}
    feeds["pos_embed"] = resample_pos_embed(np.asarray(get("pos_embed.weight")), cfg.grid,
                                            cfg.spatial_merge_size)
    feeds["rope_cos"], feeds["rope_sin"] = rope_tables(cfg)
    consts = {n for n, t in graph.tensors.items() if t.const}
    if consts != set(feeds):
        raise ValueError(f"the mapping and the graph disagree: no feed for "
                         f"{sorted(consts - set(feeds))}, no const for "
                         f"{sorted(set(feeds) - consts)}")
    for name, value in feeds.items():
        want = tuple(graph.tensors[name].shape)
        if tuple(value.shape) != want:
            raise ValueError(f"feed {name!r} has shape {tuple(value.shape)}, the graph "
                             f"declares {want}")
    return feeds
