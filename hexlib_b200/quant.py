"""q4_0 and q8_0 block quantization of weights, for staging a plan's consts.

The formats are ggml's (`block_q4_0`, `block_q8_0`; hexlib/graph/ir.py:23-41,
hexlib/exec/quant.py): blocks of 32 consecutive elements along the LAST axis,
each a little-endian fp16 scale `d` followed by the codes --

    q4_0 (18 bytes)  d = (the signed element of largest magnitude) / -8;
                     code = min(15, trunc(x / d + 8.5)) (0 when d == 0 gives
                     x * 0 + 8.5 -> 8); byte j holds element j in its low
                     nibble and element j + 16 in its high nibble;
                     value = (code - 8) * d.
    q8_0 (34 bytes)  d = max|x| / 127; code = round-half-away-from-zero of
                     x / d, saturated to int8; value = code * d.

In both the scale is narrowed to fp16 BEFORE the codes are computed, since
the codes must be correct against the scale that is stored (quant.py:85-96).
The reference builds its batch with these (wholeplan.py:293-307): a const
whose wire dtype is q4_0 is quantized from its dense value at staging, so the
backend and the numpy executor are fed the same weights.

Host-side and one-time: nothing here is on the device path.
"""
from __future__ import annotations

import numpy as np

BLOCK = 32
BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}


def nbytes(shape: tuple[int, ...], dtype: str) -> int:
    """Bytes of a block-quantized tensor (last axis a multiple of 32)."""
    if dtype not in BLOCK_BYTES:
        raise ValueError(f"{dtype!r} is not a block-quantized dtype")
    if not shape or shape[-1] % BLOCK:
        raise ValueError(f"{dtype} needs a last axis that is a multiple of {BLOCK}; "
                         f"got {tuple(shape)}")
    return int(np.prod(shape)) // BLOCK * BLOCK_BYTES[dtype]


def _blocks(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    if a.ndim == 0 or a.shape[-1] % BLOCK:
        raise ValueError(f"the last axis must be a multiple of {BLOCK}; got {a.shape}")
    return a.reshape(-1, BLOCK)


def _inverse(d16: np.ndarray) -> np.ndarray:
    du = d16.astype(np.float32)
    inv = np.zeros_like(du)
    nz = du != 0.0
    inv[nz] = np.float32(1.0) / du[nz]
    return inv


def quantize_q4_0(x: np.ndarray) -> bytes:
    b = _blocks(x)
    n = b.shape[0]
    extreme = b[np.arange(n), np.abs(b).argmax(axis=1)]
    d16 = (extreme / np.float32(-8.0)).astype(np.float32).astype(np.float16)
    scaled = b * _inverse(d16)[:, None]
    codes = np.clip(np.trunc(scaled + np.float32(8.5)), 0, 15).astype(np.uint8)
    out = np.empty((n, 18), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(n, 2)
    out[:, 2:] = codes[:, :16] | (codes[:, 16:] << 4)
    return out.tobytes()


def quantize_q8_0(x: np.ndarray) -> bytes:
    b = _blocks(x)
    n = b.shape[0]
    d16 = (np.abs(b).max(axis=1) / np.float32(127.0)).astype(np.float32).astype(np.float16)
    scaled = b * _inverse(d16)[:, None]
    codes = np.clip(np.sign(scaled) * np.floor(np.abs(scaled) + np.float32(0.5)), -128, 127)
    out = np.empty((n, 34), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(n, 2)
    out[:, 2:] = codes.astype(np.int8).view(np.uint8)
    return out.tobytes()


def quantize(x: np.ndarray, dtype: str) -> bytes:
    if dtype == "q4_0":
        return quantize_q4_0(x)
    if dtype == "q8_0":
        return quantize_q8_0(x)
    raise ValueError(f"{dtype!r} is not a block-quantized dtype")
