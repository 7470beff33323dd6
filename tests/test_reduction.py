"""Token reduction on the CPU: the restatement against the reference's own functions (golden vectors from running
them, ``tests/golden/gen_reduction_golden.py``), the product's host plan against the same vectors, the compact-order
maps, and the schedule's option rules."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from cases import REDUCTION_CASES, reduction_inputs
from oracle import reduction as orr

GOLDEN = Path(__file__).resolve().parent / "golden" / "reduction.npz"


def bf(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.int32).astype(np.uint32) << 16).view(np.float32)


@pytest.fixture(scope="module")
def red(h3b):
    return h3b.reduction


@pytest.mark.parametrize("case", sorted(REDUCTION_CASES))
def test_oracle_matches_reference(case):
    c, d = REDUCTION_CASES[case], np.load(GOLDEN)
    inp = reduction_inputs(c["grid"], c["video_start"], c["C"], c["seed"])
    m = orr.build(c["grid"], c["video_start"], inp["positions"].numpy())
    for k in ("first", "second", "parents", "pair_rows"):
        assert np.array_equal(m[k], d[f"{case}.{k}"]), k
    assert np.array_equal(m["positions"].astype(np.float32), d[f"{case}.positions"])
    x = inp["x"][0].float().numpy()
    pooled = orr.pool(x, m["first"], m["second"])
    assert np.array_equal(pooled, bf(d[f"{case}.pooled"]))
    got = orr.expand(x, bf(d[f"{case}.reduced"]), pooled, m["parents"], m["pair_rows"], c["scale"])
    assert np.array_equal(got, bf(d[f"{case}.restored"]))


@pytest.mark.parametrize("case", sorted(REDUCTION_CASES))
def test_product_plan_matches_reference(red, case):
    c, d = REDUCTION_CASES[case], np.load(GOLDEN)
    inp = reduction_inputs(c["grid"], c["video_start"], c["C"], c["seed"])
    plan = red.build_token_reduction(c["grid"], 1, 2, c["scale"], c["video_start"], inp["positions"].double())
    for k in ("first", "second", "parents", "pair_rows"):
        assert np.array_equal(getattr(plan, k).numpy(), d[f"{case}.{k}"]), k
    assert np.array_equal(plan.positions.float().numpy(), d[f"{case}.positions"])
    assert plan.reduced_grid == (c["grid"][0], c["grid"][1], (c["grid"][2] + 1) // 2)


@pytest.mark.parametrize("grid", [(3, 4, 5), (5, 8, 12), (4, 9, 7)])
def test_pair_maps_in_compact_order(red, h3b, grid):
    tile_layout = h3b.layout.tile_layout
    plan = red.build_token_reduction(grid, 0, 1)
    L, R = tile_layout(*grid), tile_layout(*plan.reduced_grid)
    m = red.pair_maps(plan, L.perm, R.perm)
    # compact -> token through the perms equals the token-order maps
    assert torch.equal(L.perm[m["ia"].long()], plan.first[R.perm])
    assert torch.equal(L.perm[m["ib"].long()], plan.second[R.perm])
    assert torch.equal(R.perm[m["par"].long()], plan.parents[L.perm])
    pair_tok = torch.zeros(L.rows, dtype=torch.bool)
    pair_tok[plan.pair_rows] = True
    assert torch.equal(m["pair"], pair_tok[L.perm])
    # pooling then expansion with a zero update and scale 1 restores every row; an odd width leaves its last column
    # unpaired and taking the reduced row
    assert int(m["pair"].sum()) == grid[0] * grid[1] * (grid[2] - grid[2] % 2)


def test_schedule_options(red):
    S = red.TokenReductionSchedule
    assert S.from_options({"enabled": False}) is None
    d = S.from_options({"enabled": True})
    assert (d.begin, d.end, d.early_steps, d.early_end, d.update_scale) == (4, 30, 4, 40, 1.0)
    assert d.end_for_step(0) == 40 and d.end_for_step(4) == 30
    s = S.from_options({"enabled": True, "blocks": "2:45", "update_scale": 0.5}, num_blocks=50)
    assert (s.begin, s.end, s.early_steps, s.early_end, s.update_scale) == (2, 45, 0, 45, 0.5)
    for bad in ({"enabled": "yes"}, {"enabled": True, "blocks": (5, 5)}, {"enabled": True, "update_scale": 3},
                {"enabled": True, "update_scale": True}, {"enabled": True, "early": (2, 20)},
                {"enabled": True, "what": 1}, {"enabled": True, "blocks": "a:b"}):
        with pytest.raises(ValueError):
            S.from_options(bad)
    with pytest.raises(ValueError, match="past the 30 DiT blocks"):
        S.from_options({"enabled": True}, num_blocks=30)
