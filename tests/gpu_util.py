"""Device plumbing for the GPU tests: torch tensors for memory and streams,
every computation through the C ABI of libhexlib_b200.so."""
from __future__ import annotations

import numpy as np

from hexlib_b200 import _lib

OK = 1


def dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty(shape, dtype):
    import torch
    td = {np.float16: torch.float16, np.float32: torch.float32}[np.dtype(dtype).type]
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return torch.empty(shape, dtype=td, device="cuda")


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def ptr(t) -> int:
    return t.data_ptr()


def stream() -> int:
    import torch
    return torch.cuda.current_stream().cuda_stream


def call(name: str, *args) -> None:
    fn = getattr(_lib.lib(), name)
    rc = fn(*args)
    assert rc == OK, f"{name} returned {rc} ({_lib.status_name(rc)})"


def call_rc(name: str, *args) -> int:
    return getattr(_lib.lib(), name)(*args)
