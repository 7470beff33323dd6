"""Sequence parallelism for the DiT block: the token dimension is sharded over ranks by whole 64-token tiles, and one
head all-to-all before self-attention (sequence -> heads) and one after (heads -> sequence) are the only exchanges.

Layouts (P ranks, H heads, Hl = H / P heads per rank, R = rows per rank):
  sequence-sharded  [H, R, ...]        this rank's rows, every head (what the prologue writes)
  head-sharded      [P, Hl, R, ...]    every rank's rows, this rank's heads; chunk p = rank p's rows. The attention
                                        kernel reads this "chunked" layout in place (h3b_vsa_fp8_ex chunks = P).
The exchanges are ``torch.distributed.all_to_all_single`` on contiguous buffers (NCCL over NVLink on B200, gloo on
CPU in the tests). FastVideo's stock path does the same Ulysses-style exchange inside DistributedAttention
(patches/fastvideo-a01c50a.patch:12-13); the reference's fused runner is single-GPU only (patch:644-645).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class SeqParallel:
    """Process-group handle plus the shard arithmetic. ``group=None`` with ``world == 1`` means no communication."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or dist.is_initialized()) else 1
        self.rank = dist.get_rank(group) if (group is not None or dist.is_initialized()) else 0

    @classmethod
    def local(cls) -> "SeqParallel":
        """One rank with no exchange, whether or not a process group is initialized."""
        sp = cls.__new__(cls)
        sp.group, sp.world, sp.rank = None, 1, 0
        return sp

    def tiles(self, n_tiles: int) -> tuple[int, int]:
        """[first, last) tile of this rank; n_tiles must split into an even count per rank."""
        if n_tiles % (2 * self.world):
            raise ValueError(f"{n_tiles} tiles do not split into an even count per rank over {self.world} ranks")
        per = n_tiles // self.world
        return self.rank * per, (self.rank + 1) * per

    def heads(self, n_heads: int) -> tuple[int, int]:
        if n_heads % self.world:
            raise ValueError(f"{n_heads} heads do not split over {self.world} ranks")
        per = n_heads // self.world
        return self.rank * per, (self.rank + 1) * per

    def _a2a(self, src: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(src)
        dist.all_to_all_single(out, src.contiguous(), group=self.group)
        return out

    def seq_to_heads(self, x: torch.Tensor) -> torch.Tensor:
        """[H, R, ...] -> [P, Hl, R, ...]: chunk p holds rank p's rows for this rank's heads."""
        if self.world == 1:
            return x.unsqueeze(0)
        H = x.shape[0]
        return self._a2a(x.reshape(self.world, H // self.world, *x.shape[1:]))

    def heads_to_seq(self, y: torch.Tensor) -> torch.Tensor:
        """[P, Hl, R, ...] (this rank's heads for every rank's rows) -> [H, R, ...] (every head for this rank's rows).
        Chunk p of the result comes from rank p, i.e. heads p*Hl .. (p+1)*Hl: heads-first order."""
        if self.world == 1:
            return y.squeeze(0)
        out = self._a2a(y)
        return out.reshape(-1, *y.shape[2:])

    def tile_stats_to_heads(self, s: torch.Tensor) -> torch.Tensor:
        """Per-tile statistics [H, n_local, ...] -> [Hl, P * n_local, ...] in global tile order (small tensors)."""
        if self.world == 1:
            return s
        got = self.seq_to_heads(s)  # [P, Hl, n_local, ...]
        return got.transpose(0, 1).reshape(got.shape[1], -1, *got.shape[3:]).contiguous()
