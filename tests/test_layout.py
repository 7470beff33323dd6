"""The layout built from FastVideo's VSA metadata against the reference's own ``_get_layout`` (golden vectors from
running it, tests/golden/gen_layout_golden.py), and against the grid-built layout on the video tiles."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from cases import LAYOUT_CASES

GOLD = Path(__file__).resolve().parent / "golden" / "layout_from_metadata.npz"


@pytest.fixture(scope="module")
def layout(h3b):
    return h3b.layout


@pytest.mark.parametrize("name", list(LAYOUT_CASES))
def test_layout_from_metadata_matches_reference(layout, name):
    gold = np.load(GOLD)
    c = LAYOUT_CASES[name]
    m = layout.vsa_metadata(tuple(c["grid"]), c["prefix"])
    lay = layout.tile_layout_from_metadata(m["untile_combined_index"], m["variable_block_sizes"])
    np.testing.assert_array_equal(lay.perm.numpy(), gold[f"{name}.perm"])
    inv = torch.empty_like(lay.perm)
    inv[lay.perm] = torch.arange(lay.rows)
    np.testing.assert_array_equal(inv.numpy(), gold[f"{name}.inv"])
    np.testing.assert_array_equal(lay.slot.numpy(), gold[f"{name}.slot"])
    n = int(gold[f"{name}.n_tiles"])
    assert lay.n_tiles == n and lay.n_ext == int(gold[f"{name}.n_ext"])
    np.testing.assert_array_equal(lay.tile_row0[:n].numpy(), gold[f"{name}.tile_row0"])
    np.testing.assert_array_equal(lay.vbs[:n].numpy(), gold[f"{name}.vbs"])
    np.testing.assert_array_equal(lay.vbs.numpy(), gold[f"{name}.vbs_ext"])
    n_pre = int(lay.vbs[:m["num_prefix_tiles"]].sum())
    assert n_pre == int(gold[f"{name}.n_pre"])


def test_video_tiles_match_grid_layout(layout):
    grid, prefix = (5, 8, 12), 100
    m = layout.vsa_metadata(grid, prefix)
    lay = layout.tile_layout_from_metadata(m["untile_combined_index"], m["variable_block_sizes"])
    g = layout.tile_layout(*grid)
    assert torch.equal(lay.perm[prefix:] - prefix, g.perm)
    n_pre = m["num_prefix_tiles"]
    assert torch.equal(lay.vbs[n_pre:n_pre + g.n_tiles], g.vbs[:g.n_tiles])


def test_metadata_with_gapped_tile_slots_is_rejected(layout):
    m = layout.vsa_metadata((2, 4, 4), 0)
    untile = m["untile_combined_index"].clone()
    untile[0] = 63  # the tile's first token moved to the last slot: the slots 0 .. vbs-1 are no longer contiguous
    with pytest.raises(ValueError, match="slots"):
        layout.tile_layout_from_metadata(untile, m["variable_block_sizes"])


def test_compute_topk(layout):
    assert layout.compute_topk(0.8, 2016) == 404
    assert layout.compute_topk(0.0, 10) == 10
    assert layout.compute_topk(0.99, 10) == 1
