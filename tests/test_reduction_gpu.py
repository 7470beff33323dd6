"""Token reduction on the GPU: the pool / expand kernels bit-exact against the reference's own functions (golden
vectors), and the runner with a reduced block interval equal, bit for bit, to the same blocks run as separate runners
on the full and the half-width grids with the pooling and expansion done by the CPU oracle in token order."""
from __future__ import annotations

import dataclasses
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import REDUCTION_CASES, reduction_inputs
from oracle import reduction as orr

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "reduction.npz"


@pytest.mark.parametrize("case", sorted(REDUCTION_CASES))
def test_pool_expand_kernels_match_reference(ops, case):
    c, d = REDUCTION_CASES[case], np.load(GOLDEN)
    inp = reduction_inputs(c["grid"], c["video_start"], c["C"], c["seed"])
    x = inp["x"][0].to(DEV)
    first = torch.from_numpy(d[f"{case}.first"]).to(DEV, torch.int32)
    second = torch.from_numpy(d[f"{case}.second"]).to(DEV, torch.int32)
    R = first.numel()
    out = torch.empty(R, x.shape[1], device=DEV, dtype=torch.bfloat16)
    pooled = torch.empty_like(out)
    ops.pool_pairs(x, first, second, out, pooled)
    want = torch.from_numpy(d[f"{case}.pooled"]).to(DEV)
    assert torch.equal(out.view(torch.int16), want) and torch.equal(pooled.view(torch.int16), want)
    reduced = torch.from_numpy(d[f"{case}.reduced"]).to(DEV).view(torch.bfloat16)
    par = torch.from_numpy(d[f"{case}.parents"]).to(DEV, torch.int32)
    pair = torch.zeros(x.shape[0], dtype=torch.bool)
    pair[torch.from_numpy(d[f"{case}.pair_rows"])] = True
    xe = x.clone()
    ops.expand_pairs(xe, reduced, pooled, par, pair.to(DEV), c["scale"])
    assert torch.equal(xe.view(torch.int16), torch.from_numpy(d[f"{case}.restored"]).to(DEV))


def test_pool_expand_large(ops, h3b):
    """124,992 x 5120 (the BASELINE latent): pooling against the oracle on every row, expansion on a row sample."""
    red = h3b.reduction
    grid = (31, 48, 84)
    plan = red.build_token_reduction(grid, 0, 1, 0.75)
    S, C = plan.parents.numel(), 5120
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(S, C, device=DEV, generator=g).bfloat16()
    out = torch.empty(plan.reduced_length, C, device=DEV, dtype=torch.bfloat16)
    pooled = torch.empty_like(out)
    ops.pool_pairs(x, plan.first.to(DEV, torch.int32), plan.second.to(DEV, torch.int32), out, pooled)
    upd = (out.float() + torch.randn(out.shape, device=DEV, generator=g) * 0.1).bfloat16()
    pair = torch.zeros(S, dtype=torch.bool)
    pair[plan.pair_rows] = True
    xe = x.clone()
    ops.expand_pairs(xe, upd, pooled, plan.parents.to(DEV, torch.int32), pair.to(DEV), 0.75)
    rows = torch.arange(0, S, 997)
    xs = x.float().cpu().numpy()
    want_pool = orr.pool(xs, plan.first.numpy(), plan.second.numpy())
    assert np.array_equal(out.float().cpu().numpy(), want_pool)
    want = orr.expand(xs, upd.float().cpu().numpy(), want_pool, plan.parents.numpy(), plan.pair_rows.numpy(), 0.75)
    assert np.array_equal(xe.float().cpu().numpy()[rows], want[rows])


def test_runner_with_reduced_interval(h3b):
    model, runner, red = h3b.model, h3b.runner, h3b.reduction
    cfg = model.DiTConfig(blocks=3)
    m = model.DiTModel.random(cfg, DEV, seed=6)
    grid = (8, 16, 24)
    g = torch.Generator(device=DEV).manual_seed(21)
    S = grid[0] * grid[1] * grid[2]
    x = torch.randn(1, S, cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    plan = red.build_token_reduction(grid, begin=1, end=2, update_scale=0.8)
    got = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx, reduction=plan)

    def sub(a, b):
        return model.DiTModel(dataclasses.replace(cfg, blocks=b - a), m.transformer_blocks[a:b], m.time_mlp,
                              m.time_proj)

    x1 = runner.H3FastRunner(sub(0, 1)).forward(x, temb, None, None, meta, context=ctx)[0].float().cpu().numpy()
    pooled = orr.pool(x1, plan.first.numpy(), plan.second.numpy())
    rmeta = dataclasses.replace(meta, grid=plan.reduced_grid)
    rot = h3b.layout.rope_positions(plan.positions)
    xr_in = torch.from_numpy(pooled).to(DEV).bfloat16()[None]
    x2 = runner.H3FastRunner(sub(1, 2)).forward(xr_in, temb, None, rot, rmeta, context=ctx)[0].float().cpu().numpy()
    x3_in = orr.expand(x1, x2, pooled, plan.parents.numpy(), plan.pair_rows.numpy(), 0.8)
    want = runner.H3FastRunner(sub(2, 3)).forward(torch.from_numpy(x3_in).to(DEV).bfloat16()[None], temb, None, None,
                                                  meta, context=ctx)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    plain = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    assert not torch.equal(got, plain)
