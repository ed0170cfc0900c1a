"""A device session: the host side of include/hexlib_b200.h's batch path.

Mirrors the reference's session lifecycle (hexlib/runtime/idl/hexlib_iface.idl:
open/start -> mmap -> invoke -> stop/close; hexlib/runtime/host/session.c):

    s = Session(device=0)
    s.load(plan, max_images=64)       # mmap both buffers, stage the consts
    out = s.run(images)               # [B, 3, 2, S, S] -> {name: [B, ...]}
    s.close()

`run` is the end-to-end call: host -> device copy of the inputs, one invoke
(one CUDA-graph launch after the first), device -> host copy of the outputs.
`invoke` alone runs on inputs already resident in HBM. Every failure raises
`B200Error` carrying the wire status; nothing falls back to another engine.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from hexlib_b200 import _lib, wire
from hexlib_b200.wholeplan import CONST_FD, IMAGE_FD, CudaPlan

MODE_GRAPH = 0
MODE_EAGER = 1


class B200Error(RuntimeError):
    def __init__(self, what: str, status: int, response: wire.BatchResponse | None = None):
        self.status = status
        self.response = response
        super().__init__(f"{what}: {wire.STATUS_NAME.get(status, status)} ({status})")


def _ok(what: str, rc: int) -> None:
    if rc != wire.STATUS["OK"]:
        raise B200Error(what, rc)


def _host_ptr(a) -> tuple[int, int]:
    """(address, nbytes) of a C-contiguous numpy array or CPU torch tensor."""
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("host array must be C-contiguous")
        return a.ctypes.data, a.nbytes
    if hasattr(a, "data_ptr") and hasattr(a, "is_contiguous"):
        if a.is_cuda or not a.is_contiguous():
            raise ValueError("host tensor must be a contiguous CPU tensor")
        return a.data_ptr(), a.numel() * a.element_size()
    raise TypeError(f"unsupported host buffer {type(a).__name__}")


@dataclass(frozen=True)
class HwInfo:
    arch: int
    sm_count: int
    hbm_bytes: int
    mapped_bytes: int


class Session:
    def __init__(self, device: int = 0) -> None:
        self._L = _lib.lib()
        h = ctypes.c_void_p()
        _ok("hexlib_b200_open", self._L.hexlib_b200_open(int(device), ctypes.byref(h)))
        self._h = h
        self.device = device
        self.plan: CudaPlan | None = None
        self.max_images = 0
        self._rsp = None
        self._blob = None

    # -- lifecycle ---------------------------------------------------------------
    def close(self) -> None:
        if self._h:
            self._L.hexlib_b200_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # noqa: D105
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def hwinfo(self) -> HwInfo:
        arch, sms = ctypes.c_uint32(), ctypes.c_uint32()
        hbm, mapped = ctypes.c_uint64(), ctypes.c_uint64()
        _ok("hwinfo", self._L.hexlib_b200_hwinfo(self._h, ctypes.byref(arch), ctypes.byref(sms),
                                                 ctypes.byref(hbm), ctypes.byref(mapped)))
        return HwInfo(arch.value, sms.value, hbm.value, mapped.value)

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _ok("stream", self._L.hexlib_b200_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    # -- buffers -------------------------------------------------------------------
    def mmap(self, fd: int, size: int, replicas: int = 1) -> None:
        _ok(f"mmap fd {fd}", self._L.hexlib_b200_mmap(self._h, fd, size, replicas))

    def munmap(self, fd: int) -> None:
        _ok(f"munmap fd {fd}", self._L.hexlib_b200_munmap(self._h, fd))

    def write(self, fd: int, offset: int, host) -> None:
        p, n = _host_ptr(host)
        _ok(f"buf_write fd {fd}", self._L.hexlib_b200_buf_write(self._h, fd, offset, p, n))

    def read(self, fd: int, offset: int, host) -> None:
        p, n = _host_ptr(host)
        _ok(f"buf_read fd {fd}", self._L.hexlib_b200_buf_read(self._h, fd, offset, p, n))

    def write_async(self, fd: int, offset: int, host) -> None:
        """Enqueue the copy on the session stream; `host` must stay valid until
        sync() and be page-locked for the copy to overlap other streams."""
        p, n = _host_ptr(host)
        _ok(f"buf_write_async fd {fd}",
            self._L.hexlib_b200_buf_write_async(self._h, fd, offset, p, n))

    def read_async(self, fd: int, offset: int, host) -> None:
        p, n = _host_ptr(host)
        _ok(f"buf_read_async fd {fd}",
            self._L.hexlib_b200_buf_read_async(self._h, fd, offset, p, n))

    def device_ptr(self, fd: int) -> tuple[int, int]:
        p, n = ctypes.c_uint64(), ctypes.c_uint64()
        _ok("buf_device_ptr", self._L.hexlib_b200_buf_device_ptr(self._h, fd, ctypes.byref(p),
                                                                 ctypes.byref(n)))
        return p.value, n.value

    # -- the plan --------------------------------------------------------------------
    def load(self, plan: CudaPlan, max_images: int = 1) -> None:
        """Register the const and per-image buffers and stage the consts."""
        if plan.const_payload is None:
            raise ValueError("plan was built without feeds; pass feeds to build_cuda_plan")
        if self.plan is not None:
            self.munmap(CONST_FD)
            self.munmap(IMAGE_FD)
        self.mmap(CONST_FD, plan.const_bytes, 1)
        self.mmap(IMAGE_FD, plan.image_bytes, max(1, int(max_images)))
        self.write(CONST_FD, 0, np.frombuffer(plan.const_payload, np.uint8))
        self.plan = plan
        self.max_images = max(1, int(max_images))
        self._blob = (ctypes.c_uint8 * len(plan.blob)).from_buffer_copy(plan.blob)
        self._rsp = (ctypes.c_uint8 * plan.response_capacity())()

    def _need(self) -> CudaPlan:
        if self.plan is None:
            raise RuntimeError("no plan loaded")
        return self.plan

    def tensor_offset(self, name: str, n_images: int) -> tuple[int, int]:
        """(byte offset in the image buffer, bytes for n images) of a tensor."""
        p = self._need().placements[name]
        if p.buffer != IMAGE_FD:
            raise ValueError(f"{name!r} is a const")
        return p.offset * n_images, p.nbytes * n_images

    def write_input(self, name: str, host, n_images: int, wait: bool = True) -> None:
        off, nb = self.tensor_offset(name, n_images)
        _, have = _host_ptr(host)
        if have != nb:
            raise ValueError(f"input {name!r} for {n_images} images is {nb} bytes, got {have}")
        (self.write if wait else self.write_async)(IMAGE_FD, off, host)

    def read_output(self, name: str, n_images: int, out=None, wait: bool = True) -> np.ndarray:
        p = self._need().placements[name]
        off, nb = self.tensor_offset(name, n_images)
        if out is None:
            out = np.empty((n_images,) + tuple(p.shape),
                           {"fp16": np.float16, "fp32": np.float32}[p.dtype])
        _, have = _host_ptr(out)
        if have != nb:
            raise ValueError(f"output {name!r} for {n_images} images is {nb} bytes, got {have}")
        (self.read if wait else self.read_async)(IMAGE_FD, off, out)
        return out

    def invoke(self, n_images: int, mode: int = MODE_GRAPH, sync: bool = True) -> wire.BatchResponse:
        plan = self._need()
        if not 1 <= n_images <= self.max_images:
            raise ValueError(f"n_images {n_images} outside 1..{self.max_images}")
        rlen = ctypes.c_uint32()
        rc = self._L.hexlib_b200_invoke_images(
            self._h, ctypes.addressof(self._blob), len(plan.blob), n_images, mode,
            1 if sync else 0, ctypes.addressof(self._rsp), len(self._rsp), ctypes.byref(rlen))
        rsp = wire.unpack_response(bytes(self._rsp[:rlen.value]))
        if rc != wire.STATUS["OK"] or not rsp.ok:
            bad = next((i for i, r in enumerate(rsp.results) if not r.ok), None)
            where = f" at op {bad} ({plan.op_names[bad]})" if bad is not None and bad < len(plan.op_names) else ""
            raise B200Error(f"invoke{where}", rc if rc != 1 else rsp.status, rsp)
        return rsp

    def sync(self) -> None:
        _ok("sync", self._L.hexlib_b200_sync(self._h))

    def run(self, images, out=None) -> np.ndarray:
        """End to end: images [B, ...] (host) -> the graph's single output [B, ...]."""
        plan = self._need()
        if len(plan.inputs) != 1 or len(plan.outputs) != 1:
            raise ValueError("run() serves single-input single-output plans; use "
                             "write_input / invoke / read_output")
        n = int(images.shape[0])
        self.write_input(plan.inputs[0], images, n)
        self.invoke(n)
        return self.read_output(plan.outputs[0], n, out)

    def device_view(self, name: str, n_images: int):
        """A torch CUDA tensor aliasing a per-image tensor's storage (for the
        NCCL gather and for device-resident benchmarking)."""
        import torch
        p = self._need().placements[name]
        base, _ = self.device_ptr(IMAGE_FD)
        off, nb = self.tensor_offset(name, n_images)
        shape = (n_images,) + tuple(p.shape)

        class _View:
            __cuda_array_interface__ = {
                "shape": shape,
                "typestr": {"fp16": "<f2", "fp32": "<f4"}[p.dtype],
                "data": (base + off, False),
                "version": 3,
                "strides": None,
            }
        return torch.as_tensor(_View(), device=f"cuda:{self.device}")


class Pipeline:
    """Back-to-back batches of one plan through `depth` sessions on one device,
    used in turn. A step's upload, graph replay and read-back are enqueued on
    its session's stream without waiting, so the copy engines move the next
    step's images (and the previous step's embeddings) while the SMs run this
    one; each session's stream keeps its own steps in order.

        pipe = Pipeline(plan, max_images=64)
        for k, batch in enumerate(batches):          # page-locked host arrays
            pipe.submit(batch, outs[k])
        pipe.drain()                                 # every outs[k] is filled

    A host array handed to submit() must stay untouched until the step is
    retired: by drain(), or by the submit() that reuses its session
    (`depth` submits later), which waits for it first. Device-side failures
    raise B200Error at that wait.
    """

    def __init__(self, plan: CudaPlan, max_images: int, device: int = 0, depth: int = 2,
                 sessions: list[Session] | None = None) -> None:
        if len(plan.inputs) != 1 or len(plan.outputs) != 1:
            raise ValueError("Pipeline serves single-input single-output plans")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.plan = plan
        self.sessions = list(sessions or [])
        self._own = len(self.sessions)
        for s in self.sessions:
            if s.plan is not plan or s.max_images < max_images:
                raise ValueError("a shared session must hold this plan for max_images")
        while len(self.sessions) < depth:
            s = Session(device)
            s.load(plan, max_images)
            self.sessions.append(s)
        self._busy = [False] * len(self.sessions)
        self._next = 0

    def submit(self, images, out) -> Session:
        """Enqueue one batch; returns the session whose stream carries it."""
        k = self._next
        s = self.sessions[k]
        if self._busy[k]:
            s.sync()
        n = int(images.shape[0])
        s.write_input(self.plan.inputs[0], images, n, wait=False)
        self._busy[k] = True
        s.invoke(n, sync=False)
        s.read_output(self.plan.outputs[0], n, out, wait=False)
        self._next = (k + 1) % len(self.sessions)
        return s

    def drain(self) -> None:
        for k, s in enumerate(self.sessions):
            if self._busy[k]:
                self._busy[k] = False
                s.sync()

    def close(self) -> None:
        """Close the sessions this pipeline opened (not ones it was handed)."""
        for s in self.sessions[self._own:]:
            s.close()


def attention_available() -> bool:
    """True when the library's fused attention kernel serves calls (an empty
    call answers OK rather than ERR_NO_KERNEL)."""
    rc = _lib.lib().hexlib_b200_attention_fp16(None, None, None, None, 0, 128, 64, 1.0, None)
    return rc == wire.STATUS["OK"]
