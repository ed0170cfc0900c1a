"""hexlib_b200_matmul_epilogue_q4_0_noalloc against the workspace entry it
varies: two calls in a row, each bit-identical to the workspace entry on the
same inputs (the second on different inputs, so a stale scratch would show),
and the oversize refusal. Collected last; passes alone and after the rest."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from hexlib_b200 import quant
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def _inputs(seed, M, K, N):
    r = np.random.default_rng(seed)
    a = r.standard_normal((M, K)).astype(np.float16)
    w = (r.standard_normal((K, N)) * 0.02).astype(np.float32)
    bias = (r.standard_normal(N) * 0.02).astype(np.float32)
    return a, np.frombuffer(quant.quantize_q4_0(w), np.uint8).copy(), bias


@pytest.mark.parametrize("M,K,N,act", [(256, 768, 3072, 1), (300, 3072, 768, 0)])
def test_two_calls_in_a_row_match_the_workspace_entry(M, K, N, act):
    for seed in (11, 12):
        a, raw, bias = _inputs(seed, M, K, N)
        da, dw, db = U.dev(a), U.dev(raw), U.dev(bias)
        y0 = U.empty((M, N), np.float16)
        y1 = U.empty((M, N), np.float16)
        ws = U.empty((K * N,), np.float16)
        U.call("hexlib_b200_matmul_epilogue_q4_0", U.ptr(da), U.ptr(dw), U.ptr(db), U.ptr(y0),
               M, K, N, act, U.ptr(ws), ctypes.c_uint64(K * N * 2), U.stream())
        U.call("hexlib_b200_matmul_epilogue_q4_0_noalloc", U.ptr(da), U.ptr(dw), U.ptr(db),
               U.ptr(y1), M, K, N, act, U.stream())
        np.testing.assert_array_equal(U.host(y1), U.host(y0))
        # no bounded wait expired in either call
        assert U.call_rc("hexlib_b200_stream_status", U.stream()) == U.OK


def test_a_weight_beyond_the_fixed_scratch_is_refused():
    # 3072 x 3072 fp16 is 18 MiB > 8 MiB: ERR_VTCM_TOO_SMALL, nothing launched
    rc = U.call_rc("hexlib_b200_matmul_epilogue_q4_0_noalloc", 0, 1, 1, 0, 16, 3072, 3072, 0,
                   U.stream())
    assert rc == 11
