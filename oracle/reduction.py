"""CPU restatement of the token reduction (horizontal token pairing) -- TEST INFRASTRUCTURE ONLY.

Follows fastvideo/models/dits/minimax_h3_token_reduction.py (chronarion/fasth3-gb300): the row maps of
``build_token_reduction`` (:81-121), ``pool_token_pairs`` (:124-133) and ``expand_token_pairs`` (:136-150), in numpy on
token order. Float work is float32 with one bf16 rounding per stored row, as torch evaluates it. Pinned against the
reference's own functions run in torch (``tests/golden/gen_reduction_golden.py`` -> ``tests/golden/reduction.npz``).
"""
from __future__ import annotations

import numpy as np

from .quant import bf16_round

f32 = np.float32


def build(grid: tuple[int, int, int], video_start: int, positions: np.ndarray) -> dict[str, np.ndarray]:
    """first, second [R]; parents [S]; pair_rows; reduced positions (mean of the two sources) for the row-major
    (t, h, w) video grid after ``video_start`` unpaired rows."""
    t, h, w = grid
    rw = (w + 1) // 2
    prefix = np.arange(video_start)
    red = np.arange(t * h * rw)
    col = 2 * (red % rw)
    first_v = video_start + (red // rw) * w + col
    second_v = first_v + (col + 1 < w)
    full = np.arange(t * h * w)
    parents_v = video_start + (full // w) * rw + (full % w) // 2
    in_pair = 2 * ((full % w) // 2) + 1 < w
    first = np.concatenate([prefix, first_v])
    second = np.concatenate([prefix, second_v])
    pos = (positions[first].astype(np.float64) + positions[second].astype(np.float64)) * 0.5
    return {"first": first, "second": second, "parents": np.concatenate([prefix, parents_v]),
            "pair_rows": video_start + np.nonzero(in_pair)[0], "positions": pos}


def pool(x: np.ndarray, first: np.ndarray, second: np.ndarray) -> np.ndarray:
    """[S, C] float32 (bf16 values) -> [R, C]: bf16((x[first] + x[second]) * 0.5) in float32."""
    return bf16_round(((x[first].astype(f32) + x[second].astype(f32)).astype(f32) * f32(0.5)).astype(f32))


def expand(original: np.ndarray, reduced: np.ndarray, pooled: np.ndarray, parents: np.ndarray,
           pair_rows: np.ndarray, scale: float) -> np.ndarray:
    """[S, C]: reduced[parents], and for pair rows bf16(original + scale * (reduced - pooled)[parents]) in float32."""
    out = reduced[parents].astype(f32).copy()
    p = parents[pair_rows]
    update = (reduced[p].astype(f32) - pooled[p].astype(f32)).astype(f32)
    out[pair_rows] = bf16_round((original[pair_rows].astype(f32) + (f32(scale) * update).astype(f32)).astype(f32))
    return out
