"""ctypes access to oracle/_ref/libhexref.so: the reference's own scalar
kernels/*/baseline.c, compiled by oracle/build_ref.py. TEST INFRASTRUCTURE:
a second, independent checker and the per-kernel CPU baseline."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle.build_ref import LIB

_L = None


def available() -> bool:
    return os.path.exists(LIB)


def lib() -> ctypes.CDLL:
    global _L
    if _L is None:
        if not available():
            raise FileNotFoundError(f"{LIB} is not built; run python oracle/build_ref.py")
        _L = ctypes.CDLL(LIB)
    return _L


def _p(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


def call(name: str, *args) -> None:
    """Call `<name>_baseline` with numpy arrays (passed by pointer), ints and
    floats (float args must be given as ctypes.c_float)."""
    fn = getattr(lib(), f"{name}_baseline")
    conv = []
    for a in args:
        if isinstance(a, np.ndarray):
            conv.append(_p(a))
        elif isinstance(a, ctypes.c_float):
            conv.append(a)
        else:
            conv.append(ctypes.c_int(int(a)))
    fn.restype = None
    fn(*conv)
