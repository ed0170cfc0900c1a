"""ctypes binding of libhexlib_b200.so (the C ABI in include/hexlib_b200.h).

The library is the product: there is no Python or CPU fallback behind any
function here. If the shared object is missing, or cannot be loaded, `lib()`
raises -- loudly, naming the file -- rather than letting a caller silently
compute something else.
"""
from __future__ import annotations

import ctypes
import os
import threading

from hexlib_b200 import build as _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

c_int = ctypes.c_int
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_f = ctypes.c_float
c_vp = ctypes.c_void_p
c_u8p = ctypes.POINTER(ctypes.c_uint8)

# name -> argtypes; every entry point returns int except status_name.
_PROTOS: dict[str, list] = {
    "hexlib_b200_open": [c_int, ctypes.POINTER(c_vp)],
    "hexlib_b200_close": [c_vp],
    "hexlib_b200_hwinfo": [c_vp, ctypes.POINTER(c_u32), ctypes.POINTER(c_u32),
                           ctypes.POINTER(c_u64), ctypes.POINTER(c_u64)],
    "hexlib_b200_mmap": [c_vp, c_u32, c_u64, c_u32],
    "hexlib_b200_munmap": [c_vp, c_u32],
    "hexlib_b200_buf_write": [c_vp, c_u32, c_u64, c_vp, c_u64],
    "hexlib_b200_buf_read": [c_vp, c_u32, c_u64, c_vp, c_u64],
    "hexlib_b200_buf_write_async": [c_vp, c_u32, c_u64, c_vp, c_u64],
    "hexlib_b200_buf_read_async": [c_vp, c_u32, c_u64, c_vp, c_u64],
    "hexlib_b200_buf_device_ptr": [c_vp, c_u32, ctypes.POINTER(c_u64),
                                   ctypes.POINTER(c_u64)],
    "hexlib_b200_stream": [c_vp, ctypes.POINTER(c_vp)],
    "hexlib_b200_invoke": [c_vp, c_vp, c_u32, c_vp, c_u32,
                           ctypes.POINTER(c_u32)],
    "hexlib_b200_invoke_images": [c_vp, c_vp, c_u32, c_u32, c_u32, c_u32,
                                  c_vp, c_u32, ctypes.POINTER(c_u32)],
    "hexlib_b200_sync": [c_vp],
    "hexlib_b200_diag_wait_timeout": [c_vp, c_u32],
    "hexlib_b200_diag_wait_timeout_stream": [c_u32, c_vp],
    "hexlib_b200_stream_status": [c_vp],
    "hexlib_b200_nccl_available": [],
    "hexlib_b200_nccl_unique_id": [c_vp],
    "hexlib_b200_nccl_open": [c_vp, c_int, c_int, c_int, c_u32, ctypes.POINTER(c_vp)],
    "hexlib_b200_nccl_allgather_f16": [c_vp, c_vp, c_vp, c_u64, c_vp, c_u32],
    "hexlib_b200_nccl_wait": [c_vp, c_vp, c_u32],
    "hexlib_b200_nccl_abort": [c_vp],
    "hexlib_b200_nccl_close": [c_vp, c_u32],
    "hexlib_b200_check_batch": [c_vp, c_u32, ctypes.POINTER(c_u64), c_u32,
                                c_u32, c_vp, c_u32, ctypes.POINTER(c_u32)],
    "hexlib_b200_add_fp16": [c_vp, c_vp, c_vp, c_int, c_vp],
    "hexlib_b200_add_fp16_f32": [c_vp, c_vp, c_vp, c_int, c_vp],
    "hexlib_b200_cast_f32_f16": [c_vp, c_vp, c_int, c_vp],
    "hexlib_b200_scale_fp16": [c_vp, c_vp, c_int, c_f, c_vp],
    "hexlib_b200_layernorm_fp16": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_f,
                                   c_vp],
    "hexlib_b200_rmsnorm_fp16": [c_vp, c_vp, c_vp, c_int, c_int, c_f, c_vp],
    "hexlib_b200_softmax_fp16": [c_vp, c_vp, c_int, c_int, c_vp],
    "hexlib_b200_rope_2d_fp16": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                 c_vp],
    "hexlib_b200_transpose_th_fp16": [c_vp, c_vp, c_int, c_int, c_int, c_vp],
    "hexlib_b200_transpose_hd_fp16": [c_vp, c_vp, c_int, c_int, c_int, c_vp],
    "hexlib_b200_patchify_fp32": [c_vp, c_vp, c_int, c_int, c_int, c_int,
                                  c_int, c_int, c_int, c_int, c_vp],
    "hexlib_b200_matmul_fp16": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                                c_vp],
    "hexlib_b200_matmul_epilogue_fp16": [c_vp, c_vp, c_vp, c_vp, c_int, c_int,
                                         c_int, c_int, c_vp],
    "hexlib_b200_matmul_epilogue_q4_0": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_u64,
                                         c_vp],
    "hexlib_b200_matmul_epilogue_q8_0": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_u64,
                                         c_vp],
    "hexlib_b200_matmul_epilogue_q4_0_noalloc": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                                 c_int, c_vp],
    "hexlib_b200_dequant_q4_0_fp16": [c_vp, c_vp, c_int, c_int, c_vp],
    "hexlib_b200_dequant_q8_0_fp16": [c_vp, c_vp, c_int, c_int, c_vp],
    "hexlib_b200_matmul_epilogue_residual_fp16": [c_vp, c_vp, c_vp, c_vp, c_vp,
                                                  c_int, c_int, c_int, c_int,
                                                  c_vp],
    "hexlib_b200_attention_fp16": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                   c_f, c_vp],
    "hexlib_b200_matmul_epilogue_rope_fp16": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                                              c_vp, c_int, c_int, c_int, c_int, c_int, c_int,
                                              c_vp],
    "hexlib_b200_attention_qkv_fp16": [c_vp, c_vp, c_int, c_int, c_int, c_int, c_f, c_vp],
    "hexlib_b200_rope_qk_fp16": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp],
    "hexlib_b200_ln_stats_fp16": [c_vp, c_vp, c_int, c_int, c_f, c_vp],
    "hexlib_b200_patchify_fp16": [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                  c_int, c_vp],
    "hexlib_b200_matmul_epilogue_ln_fp16": [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                            c_int, c_vp],
    "hexlib_b200_matmul_epilogue_ln_rope_fp16": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                                                 c_vp, c_int, c_int, c_int, c_int, c_int,
                                                 c_int, c_vp],
}


class LibraryMissing(RuntimeError):
    pass


def lib_path() -> str:
    return _build.LIB_PATH


def lib(build_if_missing: bool = True) -> ctypes.CDLL:
    """The loaded library. Builds it first if it is absent and nvcc exists."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = lib_path()
        if not os.path.exists(path) and build_if_missing:
            try:
                _build.build()
            except Exception as e:  # noqa: BLE001 -- reported below
                raise LibraryMissing(
                    f"{path} is missing and building it failed: {e}") from e
        if not os.path.exists(path):
            raise LibraryMissing(
                f"{path} is missing; run `python -m hexlib_b200.build`. There "
                "is no fallback: every op of this backend runs in that library.")
        handle = ctypes.CDLL(path)
        for name, argtypes in _PROTOS.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = c_int
        handle.hexlib_b200_status_name.argtypes = [c_int]
        handle.hexlib_b200_status_name.restype = ctypes.c_char_p
        _LIB = handle
        return _LIB


def exported_names() -> tuple[str, ...]:
    return tuple(_PROTOS) + ("hexlib_b200_status_name",)


def status_name(code: int) -> str:
    return lib().hexlib_b200_status_name(int(code)).decode()
