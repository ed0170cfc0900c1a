"""The checkpoint mapping (hexlib_b200.checkpoint, the counterpart of
hexlib/models/loader.py feeds_from_params) pinned to the reference: the
reference's tiny golden parameters (tests/golden/tiny_params.npz) must map to
exactly the feeds the reference's loader produced from them
(tests/golden/tiny.npz feed::*), bit for bit."""
from __future__ import annotations

import dataclasses
import os

import numpy as np
import pytest

from hexlib_b200 import checkpoint
from hexlib_b200 import graph as G

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY = G.VitConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=128,
                   patch_size=4, temporal_patch_size=2, in_channels=3,
                   spatial_merge_size=2, out_hidden_size=32, layernorm_eps=1e-6,
                   rope_theta=10000.0, image_size=32, act_dtype="fp32", weight_dtype="fp32")


@pytest.fixture(scope="module")
def golden():
    return (np.load(os.path.join(GOLDEN, "tiny_params.npz")),
            np.load(os.path.join(GOLDEN, "tiny.npz")))


def test_the_tiny_goldens_parameters_map_to_the_references_feeds(golden):
    params, tiny = golden
    g = G.build_vision_encoder(TINY)
    feeds = checkpoint.feeds_from_params(g, TINY, lambda n: params[f"param::{n}"])
    want = {k[6:]: tiny[k] for k in tiny.files if k.startswith("feed::") and k != "feed::image"}
    assert set(feeds) == set(want)
    for name in sorted(want):
        got = np.asarray(feeds[name], np.float32)
        assert got.shape == want[name].shape, name
        assert np.array_equal(got.view(np.uint32), want[name].view(np.uint32)), name


def test_the_position_grid_is_resampled_not_copied(golden):
    params, tiny = golden
    table = params["param::pos_embed.weight"]
    assert table.shape[0] == 25 and TINY.grid == 8          # a 5x5 grid onto 8x8 patches
    out = checkpoint.resample_pos_embed(table, TINY.grid, TINY.spatial_merge_size)
    # corners of the patch grid land exactly on the grid's corners: token 0
    # is (0, 0); the last token of merge-block order is (7, 7)
    assert np.array_equal(out[0], table[0])
    assert np.array_equal(out[-1], table[24])


def test_a_wrong_or_incomplete_mapping_is_refused(golden):
    params, _ = golden
    g = G.build_vision_encoder(TINY)
    with pytest.raises(ValueError, match="no feed for"):
        checkpoint.feeds_from_params(g, dataclasses.replace(TINY, depth=1),
                                     lambda n: params[f"param::{n}"])

    def transposed(n):
        v = params[f"param::{n}"]
        return v.T if n == "merger.linear_fc2.weight" else v
    with pytest.raises(ValueError, match="w_m2"):
        checkpoint.feeds_from_params(g, TINY, transposed)
    with pytest.raises(ValueError, match="not a square grid"):
        checkpoint.resample_pos_embed(np.zeros((24, 4), np.float32), 8, 2)
