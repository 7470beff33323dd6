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


def vbs_pattern(n_tiles: int) -> torch.Tensor:
    """Variable tile sizes like the reference's test geometry (tests/test_kernels.py:21-25)."""
    vbs = torch.full((n_tiles,), 64, dtype=torch.int32)
    vbs[::10] = 16
    vbs[3::11] = 32
    vbs[0] = 16
    return vbs


def topk_inputs(heads: int, n: int, seed: int, quantize: float) -> torch.Tensor:
    """Scores [heads*n, n]; rounded to multiples of 1/quantize so that ties occur."""
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(heads * n, n, generator=g)
    return (s * quantize).round() / quantize


def prologue_inputs(heads: int, n_tiles: int, seed: int) -> dict[str, torch.Tensor]:
    """The reference test's prologue inputs (tests/test_kernels.py:40-47) on a variable-size tile geometry."""
    g = torch.Generator().manual_seed(seed)
    vbs = vbs_pattern(n_tiles)
    rows = int(vbs.sum())
    W = heads * 128
    d = {
        "q": torch.randn(rows, W, generator=g).bfloat16(), "k": torch.randn(rows, W, generator=g).bfloat16(),
        "v": torch.randn(rows, W, generator=g).bfloat16(), "s1": torch.rand(rows, generator=g) + 0.5,
        "wq": torch.randn(128, generator=g).bfloat16(), "wk": torch.randn(128, generator=g).bfloat16(),
    }
    ang = torch.rand(rows, 48, generator=g) * 6.28
    d["cos"] = torch.cat([ang.cos()] * 2, -1).bfloat16()
    d["sin"] = torch.cat([ang.sin()] * 2, -1).bfloat16()
    d["vbs"] = vbs
    d["tile_row0"] = (vbs.cumsum(0) - vbs).to(torch.int32)
    return d


def gate_inputs(heads: int, vbs: list[int], seed: int) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    vbs_t = torch.tensor(vbs, dtype=torch.int32)
    n_tiles = len(vbs)
    rows = int(vbs_t.sum())
    W = heads * 128
    slot = torch.cat([torch.arange(int(v)) + i * 64 for i, v in enumerate(vbs)]).to(torch.int32)
    return {"ob": torch.randn(1, heads, n_tiles * 64, 128, generator=g).bfloat16(),
            "g": torch.randn(rows, W, generator=g).bfloat16(), "sg": torch.rand(rows, generator=g) + 0.5,
            "oc": torch.randn(heads, n_tiles, 128, generator=g).bfloat16(), "slot": slot}


TOPK_CASES = {
    "topk_prefix_spans": dict(heads=4, n=96, seed=21, quantize=4.0, prefix=8, spans=[(8, 50, 9), (50, 96, 10)],
                              split=False),
    "topk_split": dict(heads=3, n=64, seed=22, quantize=2.0, prefix=4, spans=[(4, 64, 12)], split=True),
    "topk_c4": dict(heads=2, n=512, seed=23, quantize=0.0, prefix=0, spans=[(0, 512, 32)], split=False),
}
PROLOGUE_CASES = {"prologue8_h2": dict(heads=2, n_tiles=10, seed=24)}
GATE_CASES = {"gate5120_fp8": dict(heads=40, vbs=[16, 32], seed=25, fp4=False),
              "gate5120_fp4": dict(heads=40, vbs=[16, 32], seed=26, fp4=True)}


def lora_inputs(N: int, K: int, rank: int, seed: int, per_row: bool, big_every: int, big: float
                ) -> dict[str, torch.Tensor]:
    """A dense weight N(0, 0.02) with its FP8 grid (per-row or per-tensor amax/448) and a LoRA pair (A [rank, K],
    B [N, rank]) whose product is scaled up by ``big`` on every ``big_every``-th row, so that some rows (or the tensor)
    outgrow the grid's 5% slack and take their own scale."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    A = (torch.randn(rank, K, generator=g) * 0.05).bfloat16()
    B = (torch.randn(N, rank, generator=g) * 0.01).bfloat16()
    if big_every:
        B[::big_every] *= big
    amax = w.float().abs().amax(dim=1) if per_row else w.float().abs().amax().reshape(1)
    base = (amax / 448.0).clamp(min=1.0 / (448.0 * 512.0)).float()
    return {"w": w, "A": A, "B": B, "base_scale": base}


LORA_CASES = {
    "lora_rows": dict(N=128, K=256, rank=16, seed=31, per_row=True, big_every=7, big=40.0, strength=0.8, alpha=32.0),
    "lora_tensor_own": dict(N=64, K=256, rank=8, seed=32, per_row=False, big_every=5, big=60.0, strength=1.0,
                            alpha=8.0),
    "lora_tensor_grid": dict(N=64, K=256, rank=8, seed=33, per_row=False, big_every=0, big=1.0, strength=0.5,
                             alpha=16.0),
}


REDUCTION_CASES = {
    "red_odd_prefix": dict(grid=(3, 4, 5), video_start=3, C=64, seed=41, scale=0.7),
    "red_even": dict(grid=(2, 3, 8), video_start=0, C=128, seed=42, scale=1.0),
}


def reduction_inputs(grid: tuple[int, int, int], video_start: int, C: int, seed: int) -> dict[str, torch.Tensor]:
    """Hidden states [1, S, C] bf16 N(0, 1), float positions [S, 3] (prefix rows at t = -1), and a per-row update of
    the reduced rows N(0, 0.25) (what the reduced blocks add to the pooled stream)."""
    t, h, w = grid
    S = video_start + t * h * w
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, S, C, generator=g).bfloat16()
    tok = torch.arange(t * h * w)
    pos = torch.zeros(S, 3, dtype=torch.float32)
    pos[:video_start, 0] = -1.0
    pos[video_start:] = torch.stack([tok // (h * w), (tok // w) % h, tok % w], 1).float()
    R = video_start + t * h * ((w + 1) // 2)
    delta = (torch.randn(1, R, C, generator=g) * 0.25).bfloat16()
    return {"x": x, "positions": pos, "delta": delta}


def fp8_pack_weight(N: int, K: int, seed: int, std: float, big_rows: int, zero_rows: int) -> torch.Tensor:
    """A dense bf16 weight [N, K] ~ N(0, std) with ``big_rows`` rows scaled x300 (values past the E4M3 range of the
    tensor scale's neighbours) and ``zero_rows`` all-zero rows (the scale floor)."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * std
    rows = torch.randperm(N, generator=g)
    w[rows[:big_rows]] *= 300.0
    w[rows[big_rows:big_rows + zero_rows]] = 0.0
    return w.bfloat16()


FP8_PACK_CASES = {
    "fp8pack_small": dict(N=128, K=512, seed=51, std=0.02, big_rows=3, zero_rows=2),
    "fp8pack_3072": dict(N=32, K=3072, seed=52, std=0.02, big_rows=1, zero_rows=1),
}


# latent grids with exempt prefixes (text / audio / reference tokens ahead of the video tiles)
LAYOUT_CASES = {
    "layout_video_only": dict(grid=(3, 8, 8), prefix=0),
    "layout_partial_prefix": dict(grid=(5, 8, 12), prefix=100),
    "layout_prefix_512": dict(grid=(7, 16, 16), prefix=512),
}
