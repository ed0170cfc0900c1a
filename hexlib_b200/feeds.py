"""Seeded synthetic feeds for the vision encoder: images, weights and the
constant tables, identical for the CUDA path and the CPU oracle.

No public dataset or checkpoint is involved (none is reachable here), so the
workload is synthetic with the shapes and value ranges of the real one:

  image      [3, S, S] uniform [0, 1), normalised per channel with the CLIP
             mean/std the Qwen2-VL image processor uses, then duplicated along
             the temporal axis to [3, 2, S, S] fp32 (vit.py:125-129).
  weights    every const, drawn in sorted-name order from default_rng(seed):
             fp16 2-D weights ~N(0, 0.02) (q4_0 / q8_0 ones: the same draw, left
             dense for the batch builder to quantize); LayerNorm gains 1 + N(0, 0.02);
             biases, LayerNorm shifts and pos_embed ~N(0, 0.02) fp32.
  rope_cos/sin  the 2-D rotary tables of hexlib/models/loader.py:97-117
             (restated below), not random.
"""
from __future__ import annotations

import numpy as np

from hexlib_b200.graph import VitConfig, build_vision_encoder

CLIP_MEAN = np.array([0.48145466, 0.4578275, 0.40821073], np.float32)
CLIP_STD = np.array([0.26862954, 0.26130258, 0.27577711], np.float32)


def vision_position_ids(grid: int, merge: int) -> np.ndarray:
    """(row, col) of every token in merge-block order (loader.py:80-94)."""
    r = np.broadcast_to(np.arange(grid)[:, None], (grid, grid))
    c = np.broadcast_to(np.arange(grid)[None, :], (grid, grid))

    def blocks(a):
        return a.reshape(grid // merge, merge, grid // merge, merge).transpose(0, 2, 1, 3).ravel()

    return np.stack([blocks(r), blocks(c)], axis=-1)


def rope_tables(cfg: VitConfig) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [T, head_dim] fp32 (loader.py:97-117): inv_freq over head_dim/4
    frequencies, row and column angles side by side, the half duplicated."""
    d = cfg.head_dim
    half = d // 2
    inv = 1.0 / (cfg.rope_theta ** (np.arange(0, half, 2, dtype=np.float64) / half))
    pos = vision_position_ids(cfg.grid, cfg.spatial_merge_size).astype(np.float64)
    ang = (pos[:, :, None] * inv[None, None, :]).reshape(pos.shape[0], -1)
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def images(cfg: VitConfig, n: int, seed: int = 1) -> np.ndarray:
    """n normalised images [n, 3, T, S, S] fp32."""
    rng = np.random.default_rng(seed)
    s = cfg.image_size
    raw = rng.random((n, cfg.in_channels, s, s), dtype=np.float32)
    norm = (raw - CLIP_MEAN[None, :, None, None]) / CLIP_STD[None, :, None, None]
    out = np.empty((n, cfg.in_channels, cfg.temporal_patch_size, s, s), np.float32)
    for t in range(cfg.temporal_patch_size):
        out[:, :, t] = norm
    return out


def weights(cfg: VitConfig, seed: int = 0, graph=None) -> dict[str, np.ndarray]:
    """Every const of the encoder graph, seeded."""
    g = graph if graph is not None else build_vision_encoder(cfg)
    cos, sin = rope_tables(cfg)
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name in sorted(n for n, t in g.tensors.items() if t.const):
        t = g.tensors[name]
        if name == "rope_cos":
            out[name] = cos
        elif name == "rope_sin":
            out[name] = sin
        elif t.dtype == "fp16":
            out[name] = (rng.standard_normal(t.shape, dtype=np.float32) * 0.02).astype(np.float16)
        elif t.dtype in ("q4_0", "q8_0"):
            # the same draw as an fp16 weight, kept dense: the batch builder
            # quantizes it when it stages the plan
            out[name] = (rng.standard_normal(t.shape, dtype=np.float32) * 0.02).astype(np.float32)
        elif name.endswith("ln1_w") or name.endswith("ln2_w") or name == "m_ln_w":
            out[name] = (1.0 + rng.standard_normal(t.shape, dtype=np.float32) * 0.02).astype(np.float32)
        elif t.dtype == "fp32":
            out[name] = (rng.standard_normal(t.shape, dtype=np.float32) * 0.02).astype(np.float32)
        else:
            raise ValueError(f"no synthetic rule for const {name!r} of dtype {t.dtype}")
    return out
