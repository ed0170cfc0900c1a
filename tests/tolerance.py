"""The parity bar, written once.

Movement ops (patchify, both transposes, cast, and scale by a power of two)
must be bit-exact. Every other fp16 op must be within max-abs 2e-3 of the
oracle, OR within one fp16 rounding step of it where the value is large
enough that one step is itself wider than 2e-3 (|x| >= 4): two correct
fp32 computations that sum in a different order can land on either side of
an fp16 rounding boundary, and no kernel can promise better than that
without reproducing the oracle's summation order.
"""
from __future__ import annotations

import numpy as np

ATOL_F16 = 2e-3


def f16_ulp(x: np.ndarray) -> np.ndarray:
    return np.spacing(np.abs(np.asarray(x, np.float32)).astype(np.float16)).astype(np.float64)


def assert_close_f16(got, ref, atol: float = ATOL_F16, what: str = "", ulps: int = 1,
                     inner=None) -> float:
    """max-abs `atol`, or `ulps` fp16 rounding steps where those are wider.
    `ulps` is 1 for a single op; a fused composite that rounds twice and
    combines two rounded values (the RoPE epilogue: two GEMM outputs, each one
    step from the oracle's summation order, rotated and rounded) gets 2.

    `inner`: for a composite whose first result is itself rounded to fp16 and
    then combined (the residual epilogue: fp16(a @ w + b) + r), the oracle's
    value of that intermediate. One of its rounding steps -- at ITS magnitude,
    which may exceed the output's when the residual cancels part of it -- is
    added to the bound: a summation-order difference that flips the
    intermediate's rounding carries into the sum unchanged."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite values in the result"
    err = np.abs(got - ref)
    bound = np.maximum(atol, ulps * np.maximum(f16_ulp(ref), f16_ulp(got)))
    if inner is not None:
        bound = bound + f16_ulp(inner)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {err.size} elements outside "
            f"max(abs {atol}, {ulps} fp16 ulp); worst at {i}: got {got[i]!r}, "
            f"ref {ref[i]!r}, |diff| {err[i]:.3e}")
    return float(err.max()) if err.size else 0.0


def assert_bit_exact(got, ref, what: str = "") -> None:
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert got.dtype == ref.dtype, f"{what}: dtype {got.dtype} != {ref.dtype}"
    diff = got.view(np.uint8) != ref.view(np.uint8)
    assert not diff.any(), f"{what}: {int(diff.sum())} bytes differ"
