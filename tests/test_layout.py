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


@pytest.mark.parametrize("grid", [(31, 48, 84), (7, 16, 16), (5, 9, 13), (8, 16, 16)])
def test_balanced_order_renumbers_whole_tiles(layout, grid):
    """Every tile of the (t, h, w) layout appears once in the balanced layout, with its tokens in the same order; the
    row offsets and slots follow the new sizes; a shard keeps the source indices of its tiles."""
    ref = layout.tile_layout(*grid)
    bal = layout.balanced_order(ref)
    n = ref.n_tiles
    assert bal.n_tiles == n and bal.n_ext == ref.n_ext and bal.rows == ref.rows
    assert torch.equal(torch.sort(bal.source).values, torch.arange(n))
    assert torch.equal(bal.vbs[:n], ref.vbs[:n][bal.source])
    assert torch.equal(bal.tile_row0, (bal.vbs.cumsum(0) - bal.vbs).to(torch.int32))
    for i, t in enumerate(bal.source.tolist()):
        a, v = int(bal.tile_row0[i]), int(bal.vbs[i])
        b = int(ref.tile_row0[t])
        assert torch.equal(bal.perm[a:a + v], ref.perm[b:b + v])
        assert torch.equal(bal.slot[a:a + v], torch.arange(v, dtype=torch.int32) + i * 64)
    if bool((ref.vbs[:n] == 64).all()):
        assert torch.equal(bal.source, torch.arange(n))  # one size: the order is unchanged
    half = bal.shard(n // 2, n)
    assert torch.equal(half.source, bal.source[n // 2:])
    assert torch.equal(half.perm, bal.perm[int(bal.tile_row0[n // 2]):])


@pytest.mark.parametrize("grid", [(31, 48, 84), (5, 9, 13)])
def test_balanced_order_evens_the_shards(layout, grid):
    """Contiguous shards of the balanced order hold their share of rows to within one tile per size class. On the
    31 x 48 x 84 latent (252 tiles of 48 rows in the 3-frame last slab, all on the last rank in (t, h, w) order) the
    largest of 8 shards drops from 16128 rows to 15632 (mean 15624)."""
    for P in (1, 2, 4, 8):
        ref = layout.tile_layout(*grid, pad_to=2 * P)
        if ref.n_ext != ref.n_tiles:
            continue
        bal = layout.balanced_order(ref)
        per = ref.n_tiles // P
        rows = [int(bal.vbs[p * per:(p + 1) * per].sum()) for p in range(P)]
        classes = torch.unique(ref.vbs[:ref.n_tiles])
        assert max(rows) - ref.rows / P <= int(classes.sum()), (P, rows)
        if grid == (31, 48, 84) and P == 8:
            assert max(rows) == 15632
            assert max(int(ref.vbs[p * per:(p + 1) * per].sum()) for p in range(P)) == 16128
