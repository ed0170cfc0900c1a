"""Numpy restatement of every op the plan executor dispatches.

Each function takes the op's input arrays in the COMPUTE dtype the reference
interpreter hands its backends (float32, hexlib/exec/vtcm.py:35-41; int32 for
int32) plus the op's attrs, and returns a tuple of outputs in that compute
dtype. Rounding to the STORAGE dtype (fp16 for fp16 tensors) is not done
here: the executor does it at every op boundary, as VtcmImage.put does
(hexlib/exec/vtcm.py:90-113).

The precision of each body follows the reference exactly: float64 inside
layernorm, softmax and the GELUs (hexlib/graph/opdefs/elementwise.py:82-146),
float32 for add, scale, rope and the matmuls (elementwise.py:40-67,
structural.py:55-61 and 240-254, fused.py:44-53).
"""
from __future__ import annotations

import math
from typing import Any, Mapping

import numpy as np

F32 = np.float32

try:  # the same function as math.erf, vectorised
    from scipy.special import erf as _erf_vec
except Exception:  # noqa: BLE001
    _erf_vec = np.vectorize(math.erf, otypes=[np.float64])


# ---- elementwise.py -------------------------------------------------------

def add(arrays, attrs):
    """elementwise.py:40-46: numpy-broadcast sum, in the first input's dtype."""
    a, b = arrays
    return ((a + b).astype(a.dtype),)


def scale(arrays, attrs):
    """elementwise.py:62-67: x * factor. A float32 array times a Python float
    stays float32 under numpy's promotion rules, so this is one fp32 multiply."""
    (x,) = arrays
    return ((x * attrs["factor"]).astype(x.dtype),)


def layernorm(arrays, attrs):
    """elementwise.py:82-95: biased variance over the last axis, eps inside
    the square root, affine weight and bias; all in float64."""
    x, w, b = arrays
    xd = x.astype(np.float64)
    mu = xd.mean(axis=-1, keepdims=True)
    d = xd - mu
    var = (d * d).mean(axis=-1, keepdims=True)
    y = d / np.sqrt(var + attrs["eps"])
    return ((y * w + b).astype(x.dtype),)


def gelu_tanh(arrays, attrs):
    """elementwise.py:110-114: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    (x,) = arrays
    xd = x.astype(np.float64)
    u = math.sqrt(2.0 / math.pi) * (xd + 0.044715 * xd * xd * xd)
    return ((0.5 * xd * (1.0 + np.tanh(u))).astype(x.dtype),)


def gelu_erf(arrays, attrs):
    """elementwise.py:117-125: 0.5 x (1 + erf(x / sqrt 2)), float64."""
    (x,) = arrays
    xd = x.astype(np.float64)
    return ((0.5 * xd * (1.0 + _erf_vec(xd / math.sqrt(2.0)))).astype(x.dtype),)


def softmax(arrays, attrs):
    """elementwise.py:141-146: shift by the max along `axis`, exp, normalise;
    float64.

    Over the last axis the rows are independent, so they are computed a block
    of rows at a time: each row sees exactly the same float64 operations in
    the same order as in one whole-array pass (numpy reduces each contiguous
    row on its own), so the bits are the same, and the block's float64
    temporaries stay in cache instead of streaming gigabytes at 512^2 and
    1024^2."""
    (x,) = arrays
    ax = attrs["axis"]
    if ax in (-1, x.ndim - 1) and x.ndim >= 1 and x.size:
        rows = x.reshape(-1, x.shape[-1])
        out = np.empty(rows.shape, x.dtype)
        step = max(1, (1 << 16) // max(1, rows.shape[1]))
        for i in range(0, rows.shape[0], step):
            xd = rows[i:i + step].astype(np.float64)
            e = np.exp(xd - xd.max(axis=-1, keepdims=True))
            out[i:i + step] = e / e.sum(axis=-1, keepdims=True)
        return (out.reshape(x.shape),)
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(axis=ax, keepdims=True))
    return ((e / e.sum(axis=ax, keepdims=True)).astype(x.dtype),)


# ---- structural.py ---------------------------------------------------------

def matmul(arrays, attrs):
    """structural.py:55-61: batched a @ b, float32."""
    a, b = arrays
    return ((a @ b).astype(a.dtype),)


def cast(arrays, attrs):
    """structural.py:81-82: the oracle feeds every fp16 value as float32
    (hexlib/graph/eager.py:24-29), so the cast itself is a float32 copy; the
    rounding to fp16 happens when the result is stored."""
    (x,) = arrays
    if attrs["dtype"] == "int32":
        return (x.astype(np.int32),)
    return (x.astype(F32),)


def transpose(arrays, attrs):
    """structural.py:107-112."""
    (x,) = arrays
    return (np.transpose(x, tuple(attrs["perm"])),)


def reshape(arrays, attrs):
    """structural.py:131-138."""
    (x,) = arrays
    return (x.reshape(tuple(attrs["shape"])),)


def patchify(arrays, attrs):
    """structural.py:172-207: [C, T, H, W] -> [gh*gw, C*T*p*p], tokens in
    merge-block order (bh, bw, mh, mw), features in (c, t, ph, pw) order.

    Written as the scalar index map of kernels/patchify_fp32/kernel_api.h:18-38
    rather than as a reshape chain, so it is a second derivation of the same
    permutation.
    """
    (img,) = arrays
    c, t, h, w = img.shape
    p = int(attrs["patch"])
    m = int(attrs["merge"])
    gh, gw = int(attrs["grid_h"]), int(attrs["grid_w"])
    tok = np.arange(gh * gw)
    mw = tok % m
    mh = (tok // m) % m
    bw = (tok // (m * m)) % (gw // m)
    bh = tok // (m * m * (gw // m))
    row0 = (bh * m + mh) * p          # first pixel row of each token's patch
    col0 = (bw * m + mw) * p
    feat = np.arange(c * t * p * p)
    pw = feat % p
    ph = (feat // p) % p
    tt = (feat // (p * p)) % t
    cc = feat // (p * p * t)
    rows = row0[:, None] + ph[None, :]
    cols = col0[:, None] + pw[None, :]
    out = img[cc[None, :], tt[None, :], rows, cols]
    return (out.astype(img.dtype),)


def rope_2d(arrays, attrs):
    """structural.py:240-254: split-half rotation in float32,
    x*cos + concat(-x[..., D/2:], x[..., :D/2])*sin, tables indexed by token
    and broadcast over heads."""
    x, cos, sin = arrays
    xf = x.astype(F32)
    cf = cos.astype(F32)[:, None, :]
    sf = sin.astype(F32)[:, None, :]
    h = xf.shape[-1] // 2
    rot = np.concatenate([-xf[..., h:], xf[..., :h]], axis=-1)
    return ((xf * cf + rot * sf).astype(x.dtype),)


# ---- fused.py ---------------------------------------------------------------

ACTS = ("none", "gelu_tanh", "gelu_erf")


def matmul_epilogue(arrays, attrs):
    """fused.py:44-53: (a @ w + bias) in float32, cast to the activation's
    dtype, THEN the activation's own reference -- bias before activation."""
    a, w, bias = arrays
    out = (a @ w + bias).astype(a.dtype)
    act = attrs.get("act", "none")
    if act == "none":
        return (out,)
    return {"gelu_tanh": gelu_tanh, "gelu_erf": gelu_erf}[act]((out,), {})


# ---- kernels the op registry has no kind for --------------------------------

def rmsnorm(arrays, attrs):
    """kernels/rmsnorm_fp16/kernel_api.h:8-14 and baseline.c:6-19: mean of
    squares accumulated in float, inv = 1/sqrt(ms + eps), y = x * inv * w."""
    x, w = arrays
    xf = x.astype(F32)
    ms = (xf.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(F32)
    inv = F32(1.0) / np.sqrt(ms + F32(attrs["eps"]))
    return ((xf * inv * w.astype(F32)).astype(x.dtype),)


REFERENCES = {
    "add": add,
    "scale": scale,
    "layernorm": layernorm,
    "gelu_tanh": gelu_tanh,
    "gelu_erf": gelu_erf,
    "softmax": softmax,
    "matmul": matmul,
    "cast": cast,
    "transpose": transpose,
    "reshape": reshape,
    "patchify": patchify,
    "rope_2d": rope_2d,
    "matmul_epilogue": matmul_epilogue,
    "rmsnorm": rmsnorm,
}


def reference(kind: str):
    try:
        return REFERENCES[kind]
    except KeyError:
        raise KeyError(f"the oracle has no reference for op kind {kind!r}") from None


# ---- storage ------------------------------------------------------------------

STORAGE = {"fp32": np.float32, "fp16": np.float16, "int32": np.int32}


def _round_f16(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even fp16 -> fp32. numpy's own float16 conversion is a
    scalar loop; torch's CPU conversion is vectorised and IEEE-identical, so it
    is used when present (the result is the same bits either way)."""
    a = np.ascontiguousarray(a, dtype=F32)
    try:
        import torch
        return torch.from_numpy(a).to(torch.float16).to(torch.float32).numpy()
    except Exception:  # noqa: BLE001
        return a.astype(np.float16).astype(F32)


def store(value: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the storage dtype and read back in the compute dtype, which is
    what VtcmImage.put followed by VtcmImage.get does (vtcm.py:90-127)."""
    if dtype == "int32":
        return np.asarray(value).astype(np.int32)
    if dtype == "fp16":
        return _round_f16(np.asarray(value))
    return np.asarray(value).astype(STORAGE[dtype]).astype(F32)
