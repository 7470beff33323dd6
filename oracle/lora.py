"""CPU restatement of the LoRA helpers of FastH3's runner -- TEST INFRASTRUCTURE ONLY.

Follows fastvideo/models/dits/h3fast/__init__.py (chronarion/fasth3-gb300):

- ``lora_scale``: the side-branch / merge factor ``strength * alpha / rank`` (1 when alpha == rank), :63-73;
- ``on_grid``: a merged fp32 weight in E4M3 on the base weight's scale grid, :82-92;
- ``merge_fp8``: ``W + scale * B @ A`` in float32 then ``on_grid``, the order of ``_merged_fp8`` (:354-376).

Every step is float32 with IEEE rounding, as torch evaluates it on float32 tensors: the grid test is
``amax <= fl32(fl32(1.05 * 448) * s0)`` (a Python scalar meets a float32 tensor as a float32), a new scale is
``max(amax / 448, 1e-12)``, codes are ``e4m3(clamp(m / s, +-448))`` with round-to-nearest-even. The restatement is
pinned against the reference's own functions run in torch (``tests/golden/gen_lora_golden.py`` ->
``tests/golden/lora_on_grid.npz``).
"""
from __future__ import annotations

import numpy as np

from .quant import FP8_MAX, e4m3_encode

f32 = np.float32
GRID_SLACK = f32(1.05 * 448.0)  # fl32 of the Python product 1.05 * 448
MIN_SCALE = f32(1e-12)


def lora_scale(strength: float, alpha: float, rank: int) -> float:
    """The adapter factor of ``_adapter`` (:63-73): strength * alpha / rank, or strength when alpha == rank."""
    return strength * (float(alpha) / float(rank) if alpha != rank else 1.0)


def on_grid(merged: np.ndarray, scale: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(e4m3 bytes [N, K], float32 scale [N] or [1]) of ``merged`` (float32 [N, K]) on the grid ``scale`` (float32,
    one per row or one for the tensor)."""
    m = np.ascontiguousarray(merged, dtype=f32)
    s0 = np.asarray(scale, dtype=f32).reshape(-1)
    rows = s0.size > 1
    amax = np.abs(m).max(axis=1).astype(f32) if rows else np.abs(m).max().astype(f32).reshape(1)
    lim = (GRID_SLACK * s0).astype(f32)
    own = np.maximum((amax / FP8_MAX).astype(f32), MIN_SCALE).astype(f32)
    s = np.where(amax <= lim, s0, own).astype(f32)
    q = (m / (s[:, None] if rows else s)).astype(f32)
    return e4m3_encode(q), s


def merge_fp8(source: np.ndarray, A: np.ndarray, B: np.ndarray, scale: float,
              base_scale: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``_merged_fp8``'s arithmetic: float32 ``source + scale * (B @ A)`` (the product accumulated in float64 and
    rounded once, which bounds any float32 GEMM's order), then ``on_grid``."""
    prod = (B.astype(np.float64) @ A.astype(np.float64)) * scale
    merged = (source.astype(np.float64) + prod).astype(f32)
    return on_grid(merged, base_scale)
