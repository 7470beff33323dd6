"""Seeded input recipes of the golden cases. Shared by ``gen_golden.py`` (which runs the reference's kernels on a
B200 and stores their outputs here) and by the tests (which rebuild the same inputs and compare).

Inputs come from ``torch.Generator().manual_seed(seed)`` on the CPU, so they are identical on every machine with this
torch build. Shapes follow the reference's own test (tests/test_kernels.py:12-30: random adaLN index per row, tables
N(0, 0.3), x N(0, 9), y N(0, 1), row scales U(0.5, 1.5)) at the reference width 5376 and at BASELINE's 5120.
"""
from __future__ import annotations

import torch


def rnq_inputs(C: int, rows: int, seed: int, ntab: int = 6) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, C, generator=g) * 3).bfloat16()
    y = torch.randn(rows, C, generator=g).bfloat16()
    sy = torch.rand(rows, generator=g) + 0.5
    tabs = (torch.randn(ntab, 6 * C, generator=g) * 0.3).bfloat16()
    idx = torch.randint(0, ntab, (rows,), generator=g, dtype=torch.int32)
    nw = torch.randn(C, generator=g).bfloat16()
    return {"x": x, "y": y, "sy": sy, "tabs": tabs, "idx": idx, "nw": nw,
            "shift": tabs[:, :C], "scale": tabs[:, C:2 * C], "gate": tabs[:, 2 * C:3 * C]}


def outlier_matrix(rows: int, K: int, seed: int, frac: float, mult: float, std: float = 1.0) -> torch.Tensor:
    """N(0, std) bf16 with ``frac`` of the columns (randperm) scaled by ``mult`` (BASELINE configs 1 and 2)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g) * std
    n_out = int(round(frac * K))
    if n_out:
        cols = torch.randperm(K, generator=g)[:n_out]
        x[:, cols] *= mult
    return x.bfloat16()


# name -> (kind, params). Kept small: the fixtures hold the reference's outputs, inputs are rebuilt from the seed.
CASES = {
    "rnq5376_branch_rms_fp8": ("rnq", dict(C=5376, rows=16, seed=1, branch=True, norm=True, fp4=False)),
    "rnq5376_branch_rms_fp4": ("rnq", dict(C=5376, rows=16, seed=2, branch=True, norm=True, fp4=True)),
    "rnq5376_rms_fp8": ("rnq", dict(C=5376, rows=16, seed=3, branch=False, norm=True, fp4=False)),
    "rnq5376_branch_only": ("rnq", dict(C=5376, rows=16, seed=4, branch=True, norm=False, fp4=False)),
    "rnq5120_branch_rms_fp8": ("rnq", dict(C=5120, rows=16, seed=5, branch=True, norm=True, fp4=False)),
    "rnq5120_branch_rms_fp4": ("rnq", dict(C=5120, rows=16, seed=6, branch=True, norm=True, fp4=True)),
    "rnq5120_rms_fp4": ("rnq", dict(C=5120, rows=16, seed=7, branch=False, norm=True, fp4=True)),
    "nvfp4_tensor_x5120": ("nvfp4", dict(rows=32, K=5120, seed=8, frac=0.005, mult=30.0, std=1.0)),
    "nvfp4_tensor_w5120": ("nvfp4", dict(rows=64, K=5120, seed=9, frac=0.0, mult=1.0, std=0.02)),
}
