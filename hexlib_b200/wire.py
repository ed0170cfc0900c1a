"""The batch blob and its response: the format of hexlib/runtime/wire.py:24-234
and hexlib/runtime/skel/hexlib_dsp.h:109-182, byte for byte.

The format is kept identical on purpose -- it is the contract the CUDA
dispatcher consumes in place of the DSP's -- so the constants, the struct
layouts and the host-side refusals are the reference's. Two things are added,
both invisible to a blob the reference would build:

  * status codes 16 (ERR_CUDA), 17 (ERR_TIMEOUT) and 18 (ERR_COMM), appended
    after 15;
  * BUF_PER_IMAGE, a bit in `BufDesc.flags` (which the reference always
    writes 0) marking a buffer whose tensors exist once per image, so one
    blob serves a batch of B images.

There is still no field for an address: tensors are (buffer index, offset).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

BATCH_MAGIC = 0x424C5848  # 'HXLB'
BATCH_VERSION = 1

MAX_BUFS = 8
MAX_SRC = 6
MAX_DST = 4
MAX_PARAMS = 16
MAX_TENSORS = 512

STATUS = {
    "OK": 1, "ERR_INTERNAL": 2, "ERR_BAD_MAGIC": 3, "ERR_BAD_VERSION": 4,
    "ERR_TRUNCATED": 5, "ERR_INVAL_PARAMS": 6, "ERR_UNMAPPED": 7,
    "ERR_NO_MMAP_SLOT": 8, "ERR_MMAP_FAILED": 9, "ERR_NO_KERNEL": 10,
    "ERR_VTCM_TOO_SMALL": 11, "ERR_VTCM_RECLAIMED": 12, "ERR_REQUIRES": 13,
    "ERR_NOT_STARTED": 14, "ERR_CACHE": 15,
    # appended by this backend
    "ERR_CUDA": 16, "ERR_TIMEOUT": 17, "ERR_COMM": 18,
}
STATUS_NAME = {v: k for k, v in STATUS.items()}

DTYPE_ID = {"fp32": 0, "fp16": 1, "q4_0": 2, "int32": 3, "q8_0": 4}
LAYOUT_ID = {"row_major": 0, "tiled_32x32": 1, "q4_0_repacked": 2}

BUF_PER_IMAGE = 1

# little-endian layouts of hexlib_batch_hdr, hexlib_buf_desc, hexlib_tensor,
# hexlib_op_desc, hexlib_batch_rsp_hdr and hexlib_op_result
HDR = struct.Struct("<10I")
BUF = struct.Struct("<QQII")
TENSOR = struct.Struct("<11I")
OP = struct.Struct(f"<II{MAX_PARAMS}i{MAX_SRC}H{MAX_DST}H")
RSP_HDR = struct.Struct("<IIIIQII")
RESULT = struct.Struct("<IIQ")

HDR_SIZE, BUF_SIZE, TENSOR_SIZE = HDR.size, BUF.size, TENSOR.size
OP_SIZE, RSP_HDR_SIZE, RESULT_SIZE = OP.size, RSP_HDR.size, RESULT.size

NO_TENSOR = 0xFFFF


class WireError(Exception):
    pass


@dataclass(frozen=True)
class BufDesc:
    fd: int
    size: int
    flags: int = 0


@dataclass(frozen=True)
class TensorDesc:
    bi: int
    offset: int
    nbytes: int
    dtype: str
    layout: str
    ne: tuple[int, int, int, int]


@dataclass(frozen=True)
class OpDesc:
    kind: int
    params: tuple[int, ...] = ()
    src: tuple[int, ...] = ()
    dst: tuple[int, ...] = ()
    flags: int = 0


@dataclass(frozen=True)
class OpResult:
    kind: int
    status: int
    cycles: int

    @property
    def ok(self) -> bool:
        return self.status == STATUS["OK"]


@dataclass(frozen=True)
class BatchResponse:
    status: int
    n_ops: int
    cycles_total: int
    arch: int
    results: tuple[OpResult, ...] = field(default=())

    @property
    def ok(self) -> bool:
        return self.status == STATUS["OK"] and all(r.ok for r in self.results)


def _check(bufs, tensors, ops) -> None:
    """The host-side refusals of wire.pack_batch (wire.py:135-178)."""
    if len(bufs) > MAX_BUFS:
        raise WireError(f"{len(bufs)} buffers exceeds MAX_BUFS ({MAX_BUFS})")
    if len(tensors) > MAX_TENSORS:
        raise WireError(f"{len(tensors)} tensors exceeds {MAX_TENSORS}")
    for i, t in enumerate(tensors):
        if not 0 <= t.bi < len(bufs):
            raise WireError(f"tensor {i} names buffer {t.bi}; the batch has {len(bufs)}")
        if t.offset + t.nbytes > bufs[t.bi].size:
            raise WireError(
                f"tensor {i} ends at {t.offset + t.nbytes}, past buffer {t.bi} "
                f"({bufs[t.bi].size} bytes)")
        if t.dtype not in DTYPE_ID:
            raise WireError(f"tensor {i} has unknown dtype {t.dtype!r}")
        if t.layout not in LAYOUT_ID:
            raise WireError(f"tensor {i} has unknown layout {t.layout!r}")
    for i, op in enumerate(ops):
        if len(op.params) > MAX_PARAMS:
            raise WireError(f"op {i} has {len(op.params)} params, max {MAX_PARAMS}")
        if len(op.src) > MAX_SRC or len(op.dst) > MAX_DST:
            raise WireError(f"op {i} exceeds MAX_SRC/MAX_DST")
        if len(op.src) + len(op.dst) > MAX_BUFS:
            raise WireError(
                f"op {i} names {len(op.src)} sources + {len(op.dst)} destinations; "
                f"the kernel argument block holds {MAX_BUFS}")
        for j in tuple(op.src) + tuple(op.dst):
            if not 0 <= j < len(tensors):
                raise WireError(f"op {i} names tensor {j}, out of range")


def pack_batch(bufs, tensors, ops) -> bytes:
    """Serialise a batch: header, buffers, tensors, ops, in that order."""
    _check(bufs, tensors, ops)
    off_bufs = HDR_SIZE
    off_tensors = off_bufs + BUF_SIZE * len(bufs)
    off_ops = off_tensors + TENSOR_SIZE * len(tensors)
    total = off_ops + OP_SIZE * len(ops)
    parts = [HDR.pack(BATCH_MAGIC, BATCH_VERSION, total, len(bufs), len(tensors),
                      len(ops), off_bufs, off_tensors, off_ops, 0)]
    parts += [BUF.pack(0, b.size, b.fd, b.flags) for b in bufs]
    parts += [TENSOR.pack(t.bi, t.offset, t.nbytes, DTYPE_ID[t.dtype],
                          LAYOUT_ID[t.layout], *t.ne, 0, 0) for t in tensors]
    for op in ops:
        params = list(op.params) + [0] * (MAX_PARAMS - len(op.params))
        src = list(op.src) + [NO_TENSOR] * (MAX_SRC - len(op.src))
        dst = list(op.dst) + [NO_TENSOR] * (MAX_DST - len(op.dst))
        parts.append(OP.pack(op.kind, op.flags, *params, *src, *dst))
    blob = b"".join(parts)
    if len(blob) != total:
        raise WireError(f"packed {len(blob)} bytes, header says {total}")
    return blob


def unpack_response(raw: bytes) -> BatchResponse:
    """Parse a response, refusing anything the backend did not write
    (wire.py:211-234)."""
    if len(raw) < RSP_HDR_SIZE:
        raise WireError(f"response truncated: {len(raw)} < {RSP_HDR_SIZE} bytes")
    magic, version, status, n_ops, cycles, arch, _ = RSP_HDR.unpack_from(raw)
    if magic != BATCH_MAGIC:
        raise WireError(f"response magic 0x{magic:08x} != 0x{BATCH_MAGIC:08x}")
    if version != BATCH_VERSION:
        raise WireError(f"response version {version} != {BATCH_VERSION}")
    if status not in STATUS_NAME:
        raise WireError(f"response status {status} is not a known status")
    need = RSP_HDR_SIZE + RESULT_SIZE * n_ops
    if len(raw) < need:
        raise WireError(f"response claims {n_ops} results ({need} bytes), carries {len(raw)}")
    results = tuple(OpResult(*RESULT.unpack_from(raw, RSP_HDR_SIZE + i * RESULT_SIZE))
                    for i in range(n_ops))
    return BatchResponse(status, n_ops, cycles, arch, results)


def response_capacity(n_ops: int) -> int:
    return RSP_HDR_SIZE + RESULT_SIZE * n_ops
