"""q4_0 / q8_0 weights: the host quantizers (hexlib_b200/quant.py) and the
oracle's dequantizer against the reference's own bytes and values
(tests/golden/quant.npz, written by hexlib.exec.quant), on seeded blocks and
on the edge blocks the reference's tests construct."""
from __future__ import annotations

import os

import numpy as np
import pytest

from hexlib_b200 import quant
from oracle import quant as oq

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
Z = np.load(os.path.join(GOLDEN, "quant.npz"))


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
def test_quantizer_matches_the_reference_byte_for_byte(dtype):
    got = quant.quantize(Z["x"], dtype)
    want = Z[dtype].tobytes()
    assert len(got) == len(want) == quant.nbytes(Z["x"].shape, dtype)
    diff = np.frombuffer(got, np.uint8) != np.frombuffer(want, np.uint8)
    assert not diff.any(), f"{int(diff.sum())} bytes differ"


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
def test_oracle_dequantizer_matches_the_reference(dtype):
    got = oq.dequantize(Z[dtype].tobytes(), Z["x"].shape, dtype)
    np.testing.assert_array_equal(got, Z[f"deq_{dtype}"])


def test_the_edge_blocks_carry_what_they_were_built_for():
    x = Z["x"]
    raw4 = np.frombuffer(Z["q4_0"].tobytes(), np.uint8).reshape(-1, 18)
    raw8 = np.frombuffer(Z["q8_0"].tobytes(), np.uint8).reshape(-1, 34)
    blocks_per_row = x.shape[1] // 32
    e = 6 * blocks_per_row                       # first edge row, first block
    # exact halves with d = 1: truncation after +8.5, not banker's rounding
    assert raw4[e, :2].view(np.float16)[0] == np.float16(1.0)
    # a positive extreme gives q4_0 a NEGATIVE scale and q8_0 a positive one
    assert raw4[e + 1, :2].view(np.float16)[0] < 0
    assert raw8[e + 1, :2].view(np.float16)[0] > 0
    # all-zero blocks: scale 0, q4_0 codes 8 (0x88), q8_0 codes 0
    z4, z8 = raw4[9 * blocks_per_row:], raw8[9 * blocks_per_row:]
    assert np.all(z4[:, 2:] == 0x88) and np.all(z8[:, 2:] == 0)


def test_refusals():
    with pytest.raises(ValueError):
        quant.quantize(np.zeros((2, 40), np.float32), "q4_0")
    with pytest.raises(ValueError):
        quant.nbytes((4, 33), "q8_0")
    with pytest.raises(ValueError):
        oq.dequantize(b"\x00" * 17, (1, 32), "q4_0")
