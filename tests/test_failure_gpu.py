"""Failure detection on the GPU without a GPU fault: a bounded device-side
wait that nothing satisfies ends in HEXLIB_B200_ERR_TIMEOUT, and the session
and the CUDA context stay usable afterwards."""
from __future__ import annotations

import numpy as np
import pytest

from hexlib_b200 import _lib, wire
from hexlib_b200.session import Session
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def test_a_wait_that_never_completes_times_out_and_the_context_survives():
    L = _lib.lib()
    with Session(0) as s:
        rc = L.hexlib_b200_diag_wait_timeout(s._h, 20000)      # 20 ms limit
        assert rc == wire.STATUS["ERR_TIMEOUT"]
        # the error word was consumed: a plain sync is clean again
        s.sync()
        # and kernels still run and are right
        x = np.arange(4100, dtype=np.float32).astype(np.float16)
        dx = U.dev(x)
        y = U.empty(4100, np.float16)
        U.call("hexlib_b200_scale_fp16", U.ptr(dx), U.ptr(y), 4100, 0.5, U.stream())
        np.testing.assert_array_equal(U.host(y), (x.astype(np.float32) * 0.5).astype(np.float16))
        assert L.hexlib_b200_diag_wait_timeout(s._h, 0) == wire.STATUS["ERR_INVAL_PARAMS"]


def test_the_per_kernel_entries_report_a_timeout_through_stream_status():
    """The per-kernel entry points return once their work is queued; a bounded
    wait that expires in one of them is reported, once, by
    hexlib_b200_stream_status after the stream drains."""
    L = _lib.lib()
    st = U.stream()
    assert L.hexlib_b200_stream_status(st) == U.OK            # nothing recorded yet
    assert L.hexlib_b200_diag_wait_timeout_stream(20000, st) == U.OK   # queued
    assert L.hexlib_b200_stream_status(st) == wire.STATUS["ERR_TIMEOUT"]
    assert L.hexlib_b200_stream_status(st) == U.OK            # reported once, then cleared
    x = np.arange(2048, dtype=np.float32).astype(np.float16)
    dx = U.dev(x)
    y = U.empty(2048, np.float16)
    U.call("hexlib_b200_scale_fp16", U.ptr(dx), U.ptr(y), 2048, 2.0, st)
    assert L.hexlib_b200_stream_status(st) == U.OK
    np.testing.assert_array_equal(U.host(y), (x.astype(np.float32) * 2).astype(np.float16))
