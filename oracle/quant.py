"""oracle.quant -- TEST INFRASTRUCTURE: dequantization of q4_0 / q8_0 weights
and the matmul_epilogue they feed, restated for checking the CUDA path.

  dequantize(raw, shape, dtype)  -> fp32 values, (code - 8) * d for q4_0
      (hexlib/exec/quant.py dequantize_q4_0) and code * d for q8_0
      (dequantize_q8_0); d is the block's fp16 scale widened to fp32.
  dequantize_f16(...)            -> the same rounded to fp16, which is what
      the reference kernel multiplies with (kernels/matmul_epilogue_fp16/
      baseline.c:36-47: `(hexlib_hf)(df * (float)lo)`).
  matmul_epilogue_quant(a, raw, bias, K, N, dtype, act)
      -> fp32 result of act(a @ W16 + bias) before the fp16 store, with W16
      the fp16-rounded dequantized weight and fp32 accumulation
      (baseline.c:49-97), the activation as oracle.ops applies it.

Pinned by tests/test_quant.py against the reference's own quantizer bytes and
dequantized values (tests/golden/quant.npz).
"""
from __future__ import annotations

import numpy as np

from oracle import ops

BLOCK = 32
BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}


def dequantize(raw: bytes, shape: tuple[int, ...], dtype: str) -> np.ndarray:
    bb = BLOCK_BYTES[dtype]
    n = int(np.prod(shape))
    if n % BLOCK or len(raw) != n // BLOCK * bb:
        raise ValueError(f"{dtype} tensor of shape {tuple(shape)}: {len(raw)} bytes")
    blk = np.frombuffer(raw, np.uint8).reshape(-1, bb)
    d = blk[:, :2].copy().view(np.float16).reshape(-1).astype(np.float32)
    if dtype == "q4_0":
        qs = blk[:, 2:]
        codes = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32) - 8.0
    else:
        codes = blk[:, 2:].copy().view(np.int8).astype(np.float32)
    return (codes * d[:, None]).reshape(shape)


def dequantize_f16(raw: bytes, shape: tuple[int, ...], dtype: str) -> np.ndarray:
    return dequantize(raw, shape, dtype).astype(np.float16)


def matmul_epilogue_quant(a: np.ndarray, raw: bytes, bias: np.ndarray, K: int, N: int,
                          dtype: str, act: str = "none") -> np.ndarray:
    w = dequantize_f16(raw, (K, N), dtype).astype(np.float32)
    (out,) = ops.matmul_epilogue((np.asarray(a, np.float32), w, np.asarray(bias, np.float32)),
                                 {"act": act})
    return out
