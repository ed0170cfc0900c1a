"""The blob format is the reference's byte for byte (fixtures from
hexlib.runtime.wire.pack_batch and build_whole_plan_batch)."""
from __future__ import annotations

import os

import numpy as np
import pytest

from hexlib_b200 import wire

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
W = np.load(os.path.join(GOLDEN, "wire.npz"))

DT = {v: k for k, v in wire.DTYPE_ID.items()}
LY = {v: k for k, v in wire.LAYOUT_ID.items()}


def parse(blob: bytes):
    """Decode a blob into descriptors with this package's struct layouts."""
    h = wire.HDR.unpack_from(blob)
    magic, version, total, nb, nt, no, ob, ot, oo, flags = h
    assert magic == wire.BATCH_MAGIC and version == wire.BATCH_VERSION and total == len(blob)
    bufs = []
    for i in range(nb):
        _, size, fd, fl = wire.BUF.unpack_from(blob, ob + i * wire.BUF_SIZE)
        bufs.append(wire.BufDesc(fd, size, fl))
    tens = []
    for i in range(nt):
        bi, off, n, dt, ly, a, b, c, d, data, pad = wire.TENSOR.unpack_from(blob, ot + i * wire.TENSOR_SIZE)
        assert data == 0 and pad == 0
        tens.append(wire.TensorDesc(bi, off, n, DT[dt], LY[ly], (a, b, c, d)))
    ops = []
    for i in range(no):
        f = wire.OP.unpack_from(blob, oo + i * wire.OP_SIZE)
        kind, fl, params, src, dst = f[0], f[1], f[2:18], f[18:24], f[24:28]
        last = max([j for j, p in enumerate(params) if p != 0], default=-1)
        ops.append(wire.OpDesc(kind, tuple(params[:last + 1]),
                               tuple(s for s in src if s != 0xFFFF),
                               tuple(d for d in dst if d != 0xFFFF), fl))
    return bufs, tens, ops


def test_struct_sizes_are_the_dsp_headers():
    assert (wire.HDR_SIZE, wire.BUF_SIZE, wire.TENSOR_SIZE, wire.OP_SIZE,
            wire.RSP_HDR_SIZE, wire.RESULT_SIZE) == (40, 24, 44, 92, 32, 16)


@pytest.mark.parametrize("key", ["one_op", "tiny_whole_plan"])
def test_repacking_a_reference_blob_is_byte_identical(key):
    blob = bytes(W[key])
    assert wire.pack_batch(*parse(blob)) == blob


def test_response_fixture_unpacks():
    r = wire.unpack_response(bytes(W["response"]))
    assert (r.status, r.n_ops, r.cycles_total, r.arch) == (1, 2, 777, 75)
    assert r.results[0] == wire.OpResult(9, 1, 300)
    assert r.results[1].status == wire.STATUS["ERR_REQUIRES"] and not r.ok


def test_status_table_keeps_the_reference_numbers_and_appends():
    assert wire.STATUS["OK"] == 1 and wire.STATUS["ERR_CACHE"] == 15
    assert wire.STATUS["ERR_CUDA"] == 16 and wire.STATUS["ERR_TIMEOUT"] == 17
    assert len(set(wire.STATUS.values())) == len(wire.STATUS)


def _t(bi=0, off=0, n=16):
    return wire.TensorDesc(bi, off, n, "fp16", "row_major", (8, 1, 1, 1))


@pytest.mark.parametrize("bufs,tens,ops,msg", [
    ([wire.BufDesc(i, 64) for i in range(9)], [], [], "MAX_BUFS"),
    ([wire.BufDesc(0, 64)], [_t(bi=1)], [], "buffer"),
    ([wire.BufDesc(0, 8)], [_t()], [], "past"),
    ([wire.BufDesc(0, 64)], [wire.TensorDesc(0, 0, 16, "bf16", "row_major", (8, 1, 1, 1))], [], "dtype"),
    ([wire.BufDesc(0, 64)], [_t()], [wire.OpDesc(9, src=(0,), dst=(3,))], "out of range"),
    ([wire.BufDesc(0, 64)], [_t()], [wire.OpDesc(9, params=tuple(range(17)), src=(0,), dst=(0,))], "params"),
    ([wire.BufDesc(0, 64)], [_t()], [wire.OpDesc(9, src=(0,) * 6, dst=(0,) * 3)], "holds"),
])
def test_host_refuses_malformed_batches(bufs, tens, ops, msg):
    with pytest.raises(wire.WireError, match=msg):
        wire.pack_batch(bufs, tens, ops)


def test_unpack_refuses_what_the_backend_did_not_write():
    with pytest.raises(wire.WireError):
        wire.unpack_response(b"\0" * 32)           # a zeroed buffer is not success
    raw = bytearray(W["response"])
    raw[8:12] = (99).to_bytes(4, "little")
    with pytest.raises(wire.WireError):
        wire.unpack_response(bytes(raw))
    with pytest.raises(wire.WireError):
        wire.unpack_response(bytes(W["response"])[:40])
