"""Token layout of the DiT latent for the VSA path: the compact tile order of FastH3's runner (_get_layout,
fastvideo/models/dits/h3fast/__init__.py:183-260), built from the latent grid (``tile_layout``) or, as the reference
does, from FastVideo's VSA metadata (``tile_layout_from_metadata``: ``untile_combined_index`` and
``variable_block_sizes``, with any prefix tiles -- text, audio, references -- ahead of the video tiles).

Tokens of a T x H x W latent are grouped into 4 x 4 x 4 cubes (64-token tiles; cubes on the far edges are smaller,
e.g. 48 tokens when the last time slab has 3 frames). Tiles are ordered (t, h, w); tokens inside a tile (t, h, w).
``perm[i]`` is the token of tile-ordered row i; ``vbs[t]`` the valid rows of tile t; ``tile_row0[t]`` its first
compact row; ``slot[i] = tile(i) * 64 + offset`` the row's place in the padded heads-first attention layout. The
tile list is padded with empty tiles to a multiple of ``pad_to`` (2 x ranks, so every rank holds an even count).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

TILE = 64


@dataclass
class TileLayout:
    grid: tuple[int, int, int] | None  # None for a layout built from metadata
    perm: torch.Tensor       # int64 [rows]: tile-ordered row -> token
    vbs: torch.Tensor        # int32 [n_ext]
    tile_row0: torch.Tensor  # int32 [n_ext]
    slot: torch.Tensor       # int32 [rows]
    n_tiles: int             # real tiles
    n_ext: int               # padded tile count
    rows: int
    # int64 [n_tiles]: the (t, h, w)-order index of each tile when the tiles were reordered (``balanced_order``);
    # None in the reference order
    source: torch.Tensor | None = None

    def shard(self, first: int, last: int) -> "TileLayout":
        """The layout of tiles [first, last) as a standalone layout (rows renumbered from 0)."""
        vbs = self.vbs[first:last].clone()
        row0 = (vbs.cumsum(0) - vbs).to(torch.int32)
        r0 = int(self.tile_row0[first]) if first < len(self.tile_row0) else self.rows
        rows = int(vbs.sum())
        perm = self.perm[r0:r0 + rows].clone()
        slot = torch.cat([torch.arange(int(v)) + i * TILE for i, v in enumerate(vbs.tolist())]).to(torch.int32) \
            if rows else torch.zeros(0, dtype=torch.int32)
        real = min(max(self.n_tiles - first, 0), last - first)
        src = None if self.source is None else self.source[first:first + real].clone()
        return TileLayout(self.grid, perm, vbs, row0, slot, real, last - first, rows, src)


def tile_layout(T: int, H: int, W: int, pad_to: int = 2, cube=(4, 4, 4)) -> TileLayout:
    ct, ch, cw = cube
    nt, nh, nw = math.ceil(T / ct), math.ceil(H / ch), math.ceil(W / cw)
    tok = torch.arange(T * H * W).view(T, H, W)
    perm, vbs = [], []
    for a in range(nt):
        for b in range(nh):
            for c in range(nw):
                block = tok[a * ct:(a + 1) * ct, b * ch:(b + 1) * ch, c * cw:(c + 1) * cw].reshape(-1)
                perm.append(block)
                vbs.append(block.numel())
    n = len(vbs)
    n_ext = (n + pad_to - 1) // pad_to * pad_to
    vbs = torch.tensor(vbs + [0] * (n_ext - n), dtype=torch.int32)
    perm = torch.cat(perm)
    row0 = (vbs.cumsum(0) - vbs).to(torch.int32)
    slot = torch.cat([torch.arange(int(v)) + i * TILE for i, v in enumerate(vbs.tolist())]).to(torch.int32)
    return TileLayout((T, H, W), perm, vbs, row0, slot, n, n_ext, int(perm.numel()))


def balanced_order(layout: TileLayout) -> TileLayout:
    """The same tiles in an order that spreads the tiles of each size (valid-row count) evenly through the list, so
    that every contiguous run of tiles -- one rank's shard under sequence parallelism -- holds close to its share of
    the rows. In (t, h, w) order the smaller cubes of a latent's far edges sit together (the 48-row tiles of a
    3-frame last time slab fill the last ranks' shards), and the ranks with only full tiles bound the step.

    Each size class's k-th tile (of n in that class, in (t, h, w) order) takes the position key (k + 1/2) / n; tiles
    are ordered by key, ties by their (t, h, w) index. Empty padding tiles stay at the end. Tokens inside a tile keep
    their order, so per-tile work (quantization scales, tile means, scores of a tile pair) is unchanged; what moves is
    the tile numbering, hence the order of each query tile's selected key tiles and, for equal scores, which tile the
    top-k keeps."""
    n = layout.n_tiles
    vbs = layout.vbs[:n].to(torch.int64)
    key = torch.empty(n, dtype=torch.float64)
    for v in torch.unique(vbs).tolist():
        idx = (vbs == v).nonzero().reshape(-1)
        key[idx] = (torch.arange(idx.numel(), dtype=torch.float64) + 0.5) / idx.numel()
    order = torch.sort(key, stable=True).indices
    src = order if layout.source is None else layout.source[order]
    pad = layout.n_ext - n
    vbs_new = torch.cat([layout.vbs[:n][order], torch.zeros(pad, dtype=torch.int32)])
    row0 = (vbs_new.cumsum(0) - vbs_new).to(torch.int32)
    old0 = layout.tile_row0[:n].to(torch.int64)
    rows = torch.cat([torch.arange(int(old0[t]), int(old0[t]) + int(vbs[t])) for t in order.tolist()]) if n else \
        torch.zeros(0, dtype=torch.int64)
    perm = layout.perm[rows]
    slot = torch.cat([torch.arange(int(v)) + i * TILE for i, v in enumerate(vbs_new.tolist())]).to(torch.int32) \
        if layout.rows else torch.zeros(0, dtype=torch.int32)
    return TileLayout(layout.grid, perm, vbs_new, row0, slot, n, layout.n_ext, layout.rows, src)


def rope_3d(layout: TileLayout, rot_dims: int = 96, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [rows, rot_dims] (bf16) in tile order for rotate-half RoPE on the first ``rot_dims`` dims, the pairs
    (d, d + rot_dims/2) (the reference's RoPE form, tests/test_kernels.py:49-52). The rot_dims/2 frequencies are split
    evenly over the (t, h, w) axes."""
    T, H, W = layout.grid
    pos = torch.stack([layout.perm // (H * W), (layout.perm // W) % H, layout.perm % W], 1)
    return rope_positions(pos, rot_dims, theta)


def rope_positions(pos: torch.Tensor, rot_dims: int = 96, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [rows, rot_dims] (bf16) of rows at (t, h, w) positions ``pos`` [rows, 3] (integer grid coordinates, or
    the half-integer mean positions of token pairs), in the form of ``rope_3d``."""
    half = rot_dims // 2
    per_axis = half // 3
    ang = []
    for a in range(3):
        freqs = theta ** (-torch.arange(per_axis, dtype=torch.float64) / per_axis)
        ang.append(pos[:, a].double()[:, None] * freqs[None, :])
    a = torch.cat(ang, 1)
    a = torch.cat([a, torch.zeros(a.shape[0], half - a.shape[1], dtype=torch.float64)], 1)
    cos = torch.cat([a.cos(), a.cos()], 1)
    sin = torch.cat([a.sin(), a.sin()], 1)
    return cos.to(torch.bfloat16), sin.to(torch.bfloat16)


def tile_layout_from_metadata(untile_combined_index: torch.Tensor, variable_block_sizes: torch.Tensor,
                              pad_to: int = 2) -> TileLayout:
    """The layout the reference's ``_get_layout`` derives from FastVideo's metadata (__init__.py:194-202):
    ``perm = argsort(untile)`` (compact row -> packed row), ``slot = untile[perm]`` (compact row -> padded slot),
    ``tile_row0 = cumsum(vbs) - vbs``; the tile list padded with empty tiles to a multiple of ``pad_to`` (the
    reference pads to an even count). ``untile[packed row]`` is the token's slot ``tile * 64 + offset``; the offsets of
    a tile's tokens must be 0 .. vbs-1 (the slots the prologue writes and the gate quantizer reads)."""
    untile = untile_combined_index.reshape(-1).to(torch.int64).cpu()
    vbs = variable_block_sizes.reshape(-1).to(torch.int32).cpu()
    rows = untile.numel()
    if int(vbs.sum()) != rows:
        raise ValueError(f"variable_block_sizes sum to {int(vbs.sum())}, the index has {rows} tokens")
    if bool((vbs > TILE).any()) or bool((vbs < 0).any()):
        raise ValueError(f"variable_block_sizes must lie in [0, {TILE}]")
    perm = torch.argsort(untile)
    slot = untile[perm]
    n = vbs.numel()
    n_ext = (n + pad_to - 1) // pad_to * pad_to
    vbs_ext = torch.cat([vbs, torch.zeros(n_ext - n, dtype=torch.int32)])
    row0 = (vbs_ext.cumsum(0) - vbs_ext).to(torch.int32)
    want = torch.cat([torch.arange(int(v)) + i * TILE for i, v in enumerate(vbs.tolist())]) if rows else slot
    if not torch.equal(slot, want.to(slot.dtype)):
        raise ValueError("untile_combined_index: each tile's tokens must take the slots tile * 64 + 0 .. vbs - 1")
    return TileLayout(None, perm, vbs_ext, row0, slot.to(torch.int32), n, n_ext, rows)


def vsa_metadata(grid: tuple[int, int, int], prefix_tokens: int = 0, cube=(4, 4, 4)) -> dict:
    """FastVideo-style VSA metadata of a sequence of ``prefix_tokens`` exempt tokens (text, audio, references) followed
    by a T x H x W video latent in raster order: the prefix cut into 64-token tiles (the last one partial), the latent
    into 4 x 4 x 4 cubes (smaller on the far edges), tiles ordered prefix first, then (t, h, w).
    Returns ``untile_combined_index`` (int64 [S]: the slot tile * 64 + offset of packed token i),
    ``variable_block_sizes`` (int32 [n_tiles]), ``num_prefix_tiles`` and ``video_tile_spans`` ([(first video tile,
    n_tiles)])."""
    T, H, W = grid
    ct, ch, cw = cube
    nt, nh, nw = math.ceil(T / ct), math.ceil(H / ch), math.ceil(W / cw)
    n_pre = (prefix_tokens + TILE - 1) // TILE
    vbs = [min(TILE, prefix_tokens - TILE * i) for i in range(n_pre)]
    untile = torch.empty(prefix_tokens + T * H * W, dtype=torch.int64)
    untile[:prefix_tokens] = torch.arange(prefix_tokens)  # prefix tile i holds packed tokens 64i .. 64i + vbs - 1
    tok = torch.arange(T * H * W).view(T, H, W) + prefix_tokens
    tile = n_pre
    for a in range(nt):
        for b in range(nh):
            for c in range(nw):
                block = tok[a * ct:(a + 1) * ct, b * ch:(b + 1) * ch, c * cw:(c + 1) * cw].reshape(-1)
                untile[block] = tile * TILE + torch.arange(block.numel())
                vbs.append(block.numel())
                tile += 1
    return {"untile_combined_index": untile, "variable_block_sizes": torch.tensor(vbs, dtype=torch.int32),
            "num_prefix_tiles": n_pre, "video_tile_spans": [(n_pre, tile)]}


def compute_topk(sparsity: float, n_tiles: int) -> int:
    """Key tiles kept per query tile in a span of ``n_tiles`` at ``sparsity`` (the reference calls FastVideo's
    ``compute_topk`` here, __init__.py:443; FastVideo is not vendored, so its rounding is restated as
    ceil((1 - sparsity) * n), at least 1)."""
    return max(1, min(n_tiles, math.ceil((1.0 - float(sparsity)) * n_tiles - 1e-9)))
