"""The C-ABI library loads and exports what include/hexlib_b200.h declares,
and its host-side batch validation -- the checks every invoke runs before a
launch -- answers malformed and unsupported blobs with the reference's status
codes. No GPU and no kernel launch is involved: this is fault injection on
the host, through `hexlib_b200_check_batch`."""
from __future__ import annotations

import ctypes
import os
import re
import struct

import numpy as np
import pytest

from hexlib_b200 import _lib, graph as G, wholeplan, wire

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def declared_symbols() -> set[str]:
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"HEXLIB_B200_API\s+[\w\s\*]*?\b(hexlib_b200_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = declared_symbols()
    assert len(declared) >= 29
    for name in sorted(declared):
        assert hasattr(L, name), f"{name} is declared but not exported"
    assert declared == set(_lib.exported_names())


def test_status_names_match_the_wire_table():
    for name, code in wire.STATUS.items():
        assert _lib.status_name(code) == name
    assert _lib.status_name(0) == "UNKNOWN"


def check(blob: bytes, sizes, n_images=1, cap=None):
    L = _lib.lib()
    n_ops = wire.HDR.unpack_from(blob)[5] if len(blob) >= 40 else 0
    cap = cap if cap is not None else wire.response_capacity(min(max(n_ops, 1), 4096))
    rsp = (ctypes.c_uint8 * max(cap, 1))()
    rl = ctypes.c_uint32()
    arr = (ctypes.c_uint64 * len(sizes))(*sizes)
    b = (ctypes.c_uint8 * max(len(blob), 1)).from_buffer_copy(blob or b"\0")
    rc = L.hexlib_b200_check_batch(b, len(blob), arr, len(sizes), n_images, rsp, cap,
                                   ctypes.byref(rl))
    r = wire.unpack_response(bytes(rsp[:rl.value])) if rl.value >= 32 else None
    return rc, r


@pytest.fixture(scope="module")
def plan256():
    ep = G.compile_for_cuda(G.build_vision_encoder(G.qwen35_at(256)), attention=True,
                            residual=True)
    return wholeplan.build_cuda_plan(ep, None, alias=True)


def test_encoder_blob_validates(plan256):
    rc, r = check(plan256.blob, [plan256.const_bytes, plan256.image_bytes * 8], n_images=8)
    assert rc == 1 and r.ok and r.n_ops == plan256.n_ops and r.arch == 100


def test_images_beyond_the_buffer_are_refused(plan256):
    rc, r = check(plan256.blob, [plan256.const_bytes, plan256.image_bytes * 8], n_images=9)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] and r.n_ops == 0


def test_a_reference_q4_0_blob_validates_end_to_end():
    # build_whole_plan_batch of the tiny plan, by the reference: its
    # matmul_epilogue weights are q4_0 (the DSP spec's weight dtype), which
    # the dispatcher serves by dequantizing to fp16 ahead of the GEMM.
    blob = bytes(np.load(os.path.join(GOLDEN, "wire.npz"))["tiny_whole_plan"])
    size = wire.BUF.unpack_from(blob, 40)[1]
    rc, r = check(blob, [size])
    assert rc == 1 and r.ok
    hdr = wire.HDR.unpack_from(blob, 0)
    assert r.n_ops == hdr[5] and 5 in [x.kind for x in r.results]


def _first_matmul_weight(blob: bytes) -> int:
    """Byte offset of the TensorDesc of the first matmul_epilogue's weight."""
    hdr = wire.HDR.unpack_from(blob, 0)
    n_ops, off_tensors, off_ops = hdr[5], hdr[7], hdr[8]
    for i in range(n_ops):
        op = wire.OP.unpack_from(blob, off_ops + i * wire.OP.size)
        if op[0] == 5:
            src1 = op[2 + wire.MAX_PARAMS + 1]
            return off_tensors + src1 * wire.TENSOR.size
    raise AssertionError("no matmul_epilogue in the blob")


def test_bad_quantized_weights_are_refused():
    blob = bytes(np.load(os.path.join(GOLDEN, "wire.npz"))["tiny_whole_plan"])
    size = wire.BUF.unpack_from(blob, 40)[1]
    off = _first_matmul_weight(blob)
    # fp32 is no weight dtype (its byte count made consistent): ERR_REQUIRES
    t = wire.TENSOR.unpack_from(blob, off)
    k, n = t[5], t[6]
    assert t[1] + k * n * 4 <= size
    bad = _mutate(_mutate(blob, off + 12, "<I", wire.DTYPE_ID["fp32"]), off + 8, "<I", k * n * 4)
    rc, r = check(bad, [size])
    assert rc == wire.STATUS["ERR_REQUIRES"] and r.results[-1].kind == 5
    # a byte count that is not whole q4_0 blocks of the shape
    nbytes = struct.unpack_from("<I", blob, off + 8)[0]
    rc, r = check(_mutate(blob, off + 8, "<I", nbytes + 18), [size])
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"]


def _mutate(blob: bytes, off: int, fmt: str, value) -> bytes:
    b = bytearray(blob)
    struct.pack_into(fmt, b, off, value)
    return bytes(b)


def test_header_faults(plan256):
    sizes = [plan256.const_bytes, plan256.image_bytes]
    blob = plan256.blob
    assert check(blob[:20], sizes)[0] == wire.STATUS["ERR_TRUNCATED"]
    assert check(_mutate(blob, 0, "<I", 0xDEADBEEF), sizes)[0] == wire.STATUS["ERR_BAD_MAGIC"]
    assert check(_mutate(blob, 4, "<I", 2), sizes)[0] == wire.STATUS["ERR_BAD_VERSION"]
    assert check(_mutate(blob, 8, "<I", len(blob) + 4), sizes)[0] == wire.STATUS["ERR_TRUNCATED"]
    assert check(_mutate(blob, 12, "<I", 9), sizes)[0] == wire.STATUS["ERR_INVAL_PARAMS"]
    # n_ops so large that off_ops + n_ops * 92 wraps 32 bits: caught in 64-bit
    assert check(_mutate(blob, 20, "<I", 0x0B21642C), sizes, cap=4096)[0] == wire.STATUS["ERR_TRUNCATED"]
    # a response buffer too small for every op's result
    assert check(blob, sizes, cap=64)[0] == wire.STATUS["ERR_TRUNCATED"]
    # fewer registered buffers than the blob names
    assert check(blob, sizes[:1])[0] == wire.STATUS["ERR_UNMAPPED"]


def _op_off(blob: bytes, i: int) -> int:
    return wire.HDR.unpack_from(blob)[8] + i * wire.OP_SIZE


def _tensor_off(blob: bytes, i: int) -> int:
    return wire.HDR.unpack_from(blob)[7] + i * wire.TENSOR_SIZE


def test_op_faults_stop_at_the_first_failing_op(plan256):
    sizes = [plan256.const_bytes, plan256.image_bytes]
    blob = plan256.blob
    # unknown kind at op 3
    rc, r = check(_mutate(blob, _op_off(blob, 3), "<I", 99), sizes)
    assert rc == wire.STATUS["ERR_NO_KERNEL"] and r.n_ops == 4 and r.results[3].kind == 99
    # op 2 names a tensor out of range
    rc, r = check(_mutate(blob, _op_off(blob, 2) + 72, "<H", 600), sizes)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] and r.n_ops == 3
    # the matmul_epilogue at op 2 with an act code no kernel implements
    k = wire.OP.unpack_from(blob, _op_off(blob, 2))[0]
    assert k == 5
    rc, r = check(_mutate(blob, _op_off(blob, 2) + 8, "<i", 7), sizes)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] and r.n_ops == 3


def test_tensor_faults(plan256):
    sizes = [plan256.const_bytes, plan256.image_bytes]
    blob = plan256.blob
    src0 = wire.OP.unpack_from(blob, _op_off(blob, 0))[18]   # patchify's input
    t = _tensor_off(blob, src0)
    # declared dtype disagrees with the kernel: fp16 where patchify reads fp32
    rc, r = check(_mutate(blob, t + 12, "<I", 1), sizes)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] or rc == wire.STATUS["ERR_REQUIRES"]
    # a layout the kernel does not address
    rc, r = check(_mutate(blob, t + 16, "<I", 2), sizes)
    assert rc == wire.STATUS["ERR_REQUIRES"] and r.n_ops == 1
    # element count disagreeing with the byte count (would read past the tensor)
    rc, r = check(_mutate(blob, t + 20, "<I", 4), sizes)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] and r.n_ops == 1
    # tensor extending past its buffer
    rc, r = check(_mutate(blob, t + 4, "<I", plan256.image_bytes), sizes)
    assert rc == wire.STATUS["ERR_INVAL_PARAMS"] and r.n_ops == 1
