"""Training-free token reduction: inside an interval of blocks, every pair of horizontally adjacent video tokens is
averaged into one row, so those blocks see the latent at half width; before the first full-width block each token is
restored as its own saved value plus ``update_scale`` times the update its pair received.

Host side of fastvideo/models/dits/minimax_h3_token_reduction.py (the row maps, :81-121) and
fastvideo/configs/pipelines/minimax_h3_token_reduction.py (the schedule and its option rules, :17-83), for the
trailing ``(t, h, w)`` video grid of a packed sequence; ``pair_maps`` turns the token-order maps into the compact tile
order of the two layouts, as ``H3FastRunner._pair_maps`` does (fastvideo/models/dits/h3fast/__init__.py:262-278). The
row arithmetic runs on the GPU (``ops.pool_pairs`` / ``ops.expand_pairs``).
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch

OPTION_KEYS = frozenset({"enabled", "blocks", "early", "update_scale"})


@dataclass(frozen=True)
class TokenReductionSchedule:
    """Blocks ``begin <= i < end`` run on paired tokens; for the first ``early_steps`` denoising steps the interval
    extends to ``early_end`` (defaults: blocks 4..29, 4..39 for the first four steps)."""
    begin: int = 4
    end: int = 30
    early_steps: int = 4
    early_end: int = 40
    update_scale: float = 1.0

    @classmethod
    def from_options(cls, options: Mapping[str, Any], num_blocks: int | None = None
                     ) -> "TokenReductionSchedule | None":
        """Parses the ``h3_token_reduction`` mapping (keys enabled, blocks, early, update_scale); None when disabled.
        Raises ValueError on the inputs the reference rejects."""
        if not isinstance(options, Mapping) or options.keys() - OPTION_KEYS:
            raise ValueError(f"h3_token_reduction must be a mapping with keys from {sorted(OPTION_KEYS)}")
        enabled = options.get("enabled", False)
        if not isinstance(enabled, bool):
            raise ValueError("h3_token_reduction.enabled must be a boolean")
        if not enabled:
            return None
        begin, end = _int_pair(options.get("blocks", (cls.begin, cls.end)), "blocks")
        if not 0 <= begin < end:
            raise ValueError(f"h3_token_reduction.blocks must satisfy 0 <= BEGIN < END, got {begin}:{end}")
        default_early = (cls.early_steps, cls.early_end) if end < cls.early_end else (0, end)
        early_steps, early_end = _int_pair(options.get("early", default_early), "early")
        if early_steps < 0:
            raise ValueError("h3_token_reduction.early STEPS must be non-negative")
        if early_steps == 0:
            early_end = end
        elif early_end <= end:
            raise ValueError(f"h3_token_reduction.early END must exceed blocks END {end}, got {early_end}")
        if num_blocks is not None and max(end, early_end) > num_blocks:
            raise ValueError(f"h3_token_reduction block intervals end at {max(end, early_end)}, past the "
                             f"{num_blocks} DiT blocks")
        scale = options.get("update_scale", cls.update_scale)
        if isinstance(scale, bool) or not isinstance(scale, (int, float)) or not 0.0 <= float(scale) <= 2.0:
            raise ValueError("h3_token_reduction.update_scale must be a number in [0, 2]")
        return cls(begin, end, early_steps, early_end, float(scale))

    def end_for_step(self, step: int) -> int:
        return self.early_end if step < self.early_steps else self.end


def _int_pair(value: Any, name: str) -> tuple[int, int]:
    if isinstance(value, str):
        value = value.split(":")
    if (not isinstance(value, (list, tuple)) or len(value) != 2
            or any(isinstance(v, bool) or not isinstance(v, (int, str)) for v in value)):
        raise ValueError(f"h3_token_reduction.{name} must be two integers")
    try:
        return int(value[0]), int(value[1])
    except ValueError as e:
        raise ValueError(f"h3_token_reduction.{name} must be two integers") from e


def reduced_width(w: int) -> int:
    return (w + 1) // 2


@dataclass(frozen=True)
class TokenReduction:
    """Token-order row maps of one sequence whose video grid ``(t, h, w)`` ends it after ``video_start`` other rows.

    ``first`` / ``second``: the full rows averaged into each reduced row (equal when unpaired); ``parents``: the
    reduced row each full row restores from; ``pair_rows``: the full rows that belong to a true pair;
    ``positions``: float64 [reduced rows, 3] (t, h, w) positions, a pair at the mean of its sources."""
    begin: int
    end: int
    grid: tuple[int, int, int]
    video_start: int
    first: torch.Tensor
    second: torch.Tensor
    parents: torch.Tensor
    pair_rows: torch.Tensor
    positions: torch.Tensor
    update_scale: float = 1.0

    @property
    def reduced_grid(self) -> tuple[int, int, int]:
        t, h, w = self.grid
        return (t, h, reduced_width(w))

    @property
    def reduced_length(self) -> int:
        return int(self.first.numel())


def build_token_reduction(grid: tuple[int, int, int], begin: int, end: int, update_scale: float = 1.0,
                          video_start: int = 0, positions: torch.Tensor | None = None) -> TokenReduction:
    """Pairs columns (2c, 2c+1) of every (t, h) row of the row-major video grid; an odd width leaves the last column
    unpaired; the ``video_start`` leading rows are never paired. ``positions`` [video_start + t*h*w, 3] defaults to
    the grid coordinates (t, h, w) of the video rows (zeros before them)."""
    t, h, w = (int(v) for v in grid)
    if min(t, h, w) <= 0 or video_start < 0:
        raise ValueError(f"token reduction needs a non-empty video grid, got {grid}")
    S = video_start + t * h * w
    if positions is None:
        tok = torch.arange(t * h * w)
        positions = torch.zeros(S, 3, dtype=torch.float64)
        positions[video_start:] = torch.stack([tok // (h * w), (tok // w) % h, tok % w], 1).double()
    if positions.shape[0] != S:
        raise ValueError(f"positions hold {positions.shape[0]} rows, the sequence has {S}")
    rw = reduced_width(w)
    prefix = torch.arange(video_start, dtype=torch.long)
    red = torch.arange(t * h * rw, dtype=torch.long)
    col = 2 * (red % rw)
    first_v = video_start + (red // rw) * w + col
    has_pair = col + 1 < w
    second_v = first_v + has_pair.long()
    full = torch.arange(t * h * w, dtype=torch.long)
    fcol = full % w
    parent_v = video_start + (full // w) * rw + fcol // 2
    in_pair = 2 * (fcol // 2) + 1 < w
    first = torch.cat([prefix, first_v])
    second = torch.cat([prefix, second_v])
    pos = (positions.double().index_select(0, first) + positions.double().index_select(0, second)) * 0.5
    return TokenReduction(begin, end, (t, h, w), video_start, first, second, torch.cat([prefix, parent_v]),
                          video_start + torch.nonzero(in_pair).flatten(), pos, float(update_scale))


def pair_maps(plan: TokenReduction, full_perm: torch.Tensor, red_perm: torch.Tensor) -> dict[str, torch.Tensor]:
    """The maps between compact rows (``perm[i]`` = token of compact row i) of the full and the reduced layout:
    ``ia`` / ``ib`` int32 [reduced rows] (the two full compact rows of each reduced compact row), ``par`` int32
    [full rows] (the reduced compact row of each full compact row), ``pair`` bool [full rows]."""
    inv_full = torch.empty_like(full_perm)
    inv_full[full_perm] = torch.arange(full_perm.numel())
    inv_red = torch.empty_like(red_perm)
    inv_red[red_perm] = torch.arange(red_perm.numel())
    in_pair = torch.zeros(full_perm.numel(), dtype=torch.bool)
    in_pair[plan.pair_rows] = True
    return {"ia": inv_full.index_select(0, plan.first.index_select(0, red_perm)).to(torch.int32),
            "ib": inv_full.index_select(0, plan.second.index_select(0, red_perm)).to(torch.int32),
            "par": inv_red.index_select(0, plan.parents.index_select(0, full_perm)).to(torch.int32),
            "pair": in_pair.index_select(0, full_perm)}
