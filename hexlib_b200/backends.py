"""Per-op backends for hexlib's plan interpreter, computed on the GPU.

`interpreter_backends()` returns `{op_kind: Backend}` with the reference's
Backend signature `(tuple[np.ndarray, ...], attrs) -> tuple[np.ndarray, ...]`
(hexlib/exec/interpreter.py:35), so

    interpreter.run(compiled, feeds, backends=hexlib_b200.backends.interpreter_backends())

runs every op that has a CUDA kernel on the B200 and leaves the rest (reshape)
to the registry -- the same plug-in point `hexlib.exec.dsp.interpreter_backends`
(dsp.py:656-715) fills for the DSP. Each call selects the variant from the
op's attrs (`runner.select`), moves the inputs to the device in the dtypes
the kernel takes, runs the kernel through its C-ABI entry point, and returns
the result in the interpreter's compute dtype (float32).

The interpreter hands backends float32 arrays whatever the tensors' storage
dtype. Values stored as fp16 are exactly representable, so narrowing them back
to fp16 is exact; `add`'s right operand is always passed as fp32 so an fp32
pos_embed is added exactly as the interpreter adds it. Weights of
`matmul_epilogue` are consumed as fp16: a graph declaring q4_0 weights is
refused, as the kernel has no q4_0 path.
"""
from __future__ import annotations

from typing import Any, Callable, Mapping

import numpy as np

from hexlib_b200 import _lib, runner

Backend = Callable[[tuple, Mapping[str, Any]], tuple]


class BackendError(RuntimeError):
    pass


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise BackendError("no CUDA device: the CUDA backends have no CPU path")
    return torch


def _dev(a: np.ndarray, dtype):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=dtype))).cuda()


def _call(name: str, *args) -> None:
    rc = getattr(_lib.lib(), name)(*args)
    if rc != 1:
        raise BackendError(f"{name} returned {_lib.status_name(rc)} ({rc})")


def _run(kind: str, arrays: tuple, attrs: Mapping[str, Any]) -> np.ndarray:
    torch = _torch()
    vname, spec = runner.select(kind, dict(attrs))
    spec.check_requires(dict(attrs))
    s = torch.cuda.current_stream().cuda_stream
    f16, f32 = np.float16, np.float32
    if vname == "add":
        a, b = arrays
        if a.shape != b.shape:
            raise BackendError(f"add of {a.shape} and {b.shape}: the kernel adds equal shapes")
        da, db = _dev(a, f16), _dev(b, f32)
        y = torch.empty(a.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_add_fp16_f32", da.data_ptr(), db.data_ptr(), y.data_ptr(), a.size, s)
    elif vname == "cast":
        (x,) = arrays
        dx = _dev(x, f32)
        y = torch.empty(x.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_cast_f32_f16", dx.data_ptr(), y.data_ptr(), x.size, s)
    elif vname == "scale":
        (x,) = arrays
        dx = _dev(x, f16)
        y = torch.empty(x.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_scale_fp16", dx.data_ptr(), y.data_ptr(), x.size,
              float(np.float32(attrs["factor"])), s)
    elif vname == "layernorm":
        x, w, b = arrays
        R, C = int(np.prod(x.shape[:-1])), int(x.shape[-1])
        dx, dw, db = _dev(x, f16), _dev(w, f32), _dev(b, f32)
        y = torch.empty(x.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_layernorm_fp16", dx.data_ptr(), dw.data_ptr(), db.data_ptr(),
              y.data_ptr(), R, C, float(attrs["eps"]), s)
    elif vname == "softmax":
        (x,) = arrays
        C = int(x.shape[-1])
        dx = _dev(x, f16)
        y = torch.empty(x.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_softmax_fp16", dx.data_ptr(), y.data_ptr(), x.size // C, C, s)
    elif vname == "rope_2d":
        x, c, sn = arrays
        T, H, D = x.shape
        dx, dc, ds = _dev(x, f16), _dev(c, f32), _dev(sn, f32)
        y = torch.empty(x.shape, dtype=torch.float16, device="cuda")
        _call("hexlib_b200_rope_2d_fp16", dx.data_ptr(), dc.data_ptr(), ds.data_ptr(),
              y.data_ptr(), T, H, D, s)
    elif vname == "transpose":
        (x,) = arrays
        T, H, D = x.shape
        dx = _dev(x, f16)
        y = torch.empty((H, T, D), dtype=torch.float16, device="cuda")
        _call("hexlib_b200_transpose_th_fp16", dx.data_ptr(), y.data_ptr(), T, H, D, s)
    elif vname == "transpose_hd":
        (x,) = arrays
        B, T, D = x.shape
        dx = _dev(x, f16)
        y = torch.empty((B, D, T), dtype=torch.float16, device="cuda")
        _call("hexlib_b200_transpose_hd_fp16", dx.data_ptr(), y.data_ptr(), B, T, D, s)
    elif vname == "patchify":
        (img,) = arrays
        C, T, H, W = img.shape
        p, m = int(attrs["patch"]), int(attrs["merge"])
        gh, gw = int(attrs["grid_h"]), int(attrs["grid_w"])
        di = _dev(img, f32)
        y = torch.empty((gh * gw, C * T * p * p), dtype=torch.float32, device="cuda")
        _call("hexlib_b200_patchify_fp32", di.data_ptr(), y.data_ptr(), C, T, H, W, p, m,
              gh, gw, s)
    elif vname == "matmul":
        a, b = arrays
        if a.ndim != 3 or b.ndim != 3 or a.shape[0] != b.shape[0]:
            raise BackendError(f"matmul of {a.shape} @ {b.shape}: the kernel is batched 3-D")
        Bn, M, K = a.shape
        N = b.shape[2]
        da, db = _dev(a, f16), _dev(b, f16)
        y = torch.empty((Bn, M, N), dtype=torch.float16, device="cuda")
        _call("hexlib_b200_matmul_fp16", da.data_ptr(), db.data_ptr(), y.data_ptr(), Bn, M,
              K, N, s)
    elif vname == "matmul_epilogue":
        a, w, bias = arrays
        M, K = int(np.prod(a.shape[:-1])), int(a.shape[-1])
        N = int(w.shape[-1])
        code = dict(runner.ACT_CODES)[attrs.get("act", "none")]
        da, dw, db = _dev(a, f16), _dev(w, f16), _dev(bias, f32)
        y = torch.empty(a.shape[:-1] + (N,), dtype=torch.float16, device="cuda")
        _call("hexlib_b200_matmul_epilogue_fp16", da.data_ptr(), dw.data_ptr(),
              db.data_ptr(), y.data_ptr(), M, K, N, code, s)
    else:
        raise BackendError(f"no per-op backend for variant {vname!r}")
    torch.cuda.current_stream().synchronize()
    return y.cpu().numpy().astype(np.float32)


COMPUTE_KINDS = ("add", "cast", "layernorm", "matmul", "matmul_epilogue", "patchify",
                 "rope_2d", "scale", "softmax", "transpose")


def interpreter_backends(kinds=None) -> dict[str, Backend]:
    """`{kind: Backend}` for every op kind with a CUDA kernel (or the subset
    `kinds`), resolving the variant per call from the op's attrs."""
    wanted = COMPUTE_KINDS if kinds is None else [k for k in kinds if k in COMPUTE_KINDS]
    _lib.lib()  # fail now, not at the first op, if the library is missing

    def make(kind):
        def backend(arrays, attrs):
            return (_run(kind, tuple(np.asarray(a) for a in arrays), attrs),)
        return backend

    return {k: make(k) for k in wanted}
