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


# ------------------------------------------------------------------------------------------------- peer transport
class _DeviceBytes:
    """A raw device range exposed through ``__cuda_array_interface__`` so torch wraps it without copying; the tensor
    keeps this object (and through it the arena) alive."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2}
        self._owner = owner


def _align(n: int, a: int = 512) -> int:
    return (n + a - 1) // a * a


class PeerArena:
    """One device allocation per rank, mapped by every rank of the group (CUDA IPC over NVLink): named regions at the
    same offsets on every rank, then ``flag_slots`` x world flag words (slot s, sender q at word s * world + q).
    Collective: every rank constructs it with the same regions, in the same order."""

    def __init__(self, sp: SeqParallel, device, regions: dict, flag_slots: int):
        import ctypes

        from ._lib import call
        self._call = call
        self.world, self.rank = sp.world, sp.rank
        self.device = torch.device(device)
        self.offsets: dict[str, tuple[int, tuple, torch.dtype]] = {}
        off = 0
        for name, (shape, dtype) in regions.items():
            n = 1
            for s in shape:
                n *= int(s)
            self.offsets[name] = (off, tuple(shape), dtype)
            off = _align(off + n * torch.empty(0, dtype=dtype).element_size())
        self.flag_off = off
        self.flag_slots = flag_slots
        self.nbytes = off + _align(flag_slots * self.world * 4)
        self.base = 0
        self.bases = [0] * self.world
        self._opened: list[int] = []
        # every rank takes both collectives below whatever fails locally, so a failure on one rank is a failure on all
        # (and no rank is left waiting in a collective the others skipped)
        err, mine = None, None
        try:
            ptr = ctypes.c_void_p()
            call("h3b_peer_alloc", self.device.index, self.nbytes, ctypes.byref(ptr))
            self.base = int(ptr.value)
            h = (ctypes.c_ubyte * 64)()
            call("h3b_peer_export", self.base, h)
            mine = (bytes(h), self.nbytes)
        except Exception as exc:  # noqa: BLE001 -- reported to every rank below
            err = f"rank {self.rank}: {exc}"
        got: list = [None] * self.world
        dist.all_gather_object(got, mine, group=sp.group)
        if err is None:
            try:
                if any(g is None for g in got) or any(g[1] != self.nbytes for g in got):
                    raise RuntimeError("a rank has no arena, or the arena sizes differ over the ranks")
                for p, (hb, _) in enumerate(got):
                    if p == self.rank:
                        self.bases[p] = self.base
                        continue
                    peer = ctypes.c_void_p()
                    call("h3b_peer_open", (ctypes.c_ubyte * 64).from_buffer_copy(hb), ctypes.byref(peer))
                    self.bases[p] = int(peer.value)
                    self._opened.append(self.bases[p])
            except Exception as exc:  # noqa: BLE001
                err = f"rank {self.rank}: {exc}"
        errs: list = [None] * self.world
        dist.all_gather_object(errs, err, group=sp.group)
        errs = [e for e in errs if e]
        if errs:
            self._release()
            raise RuntimeError("peer arena: " + "; ".join(errs))
        raw = torch.as_tensor(_DeviceBytes(self.base, self.nbytes, self), device=self.device)
        self.tensors = {name: raw[o:o + _nbytes(shape, dt)].view(dt).view(shape)
                        for name, (o, shape, dt) in self.offsets.items()}
        self.flags = raw[self.flag_off:self.flag_off + flag_slots * self.world * 4].view(torch.int32)

    def ptr(self, p: int, name: str, byte_offset: int = 0) -> int:
        """Address of region ``name`` of rank p's allocation, as mapped in this process."""
        return self.bases[p] + self.offsets[name][0] + byte_offset

    def flag(self, p: int, slot: int, sender: int) -> int:
        return self.bases[p] + self.flag_off + 4 * (slot * self.world + sender)

    def _release(self) -> None:
        for q in self._opened:
            self._call("h3b_peer_close", q)
        self._opened = []
        if self.base:
            self._call("h3b_peer_free", self.base)
            self.base = 0

    def close(self, group=None) -> None:
        """Unmaps the peers' allocations and frees this one; collective (no rank frees while another still maps it)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        for q in self._opened:
            self._call("h3b_peer_close", q)
        self._opened = []
        dist.barrier(group=group)
        self.tensors, self.flags = {}, None
        if self.base:
            self._call("h3b_peer_free", self.base)
            self.base = 0


def _nbytes(shape, dtype) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n * torch.empty(0, dtype=dtype).element_size()


def peer_copy_plan(kind: str, r: int, p: int, g: int, dims: dict) -> tuple[int, int, int, int, int, int]:
    """Byte geometry of one chunk of the head exchange sent by rank r to rank p (group g): (src offset, src pitch,
    dst offset, dst pitch, width, height), offsets relative to the source tensor and the destination region.

    ``dims``: P ranks, H heads, G head groups of Hg = H / (P G) heads, R padded rows per rank, D = 128, n tiles per rank,
    es the element size; per kind:
      "qkv":   src [planes, H, R, D] (heads p*Hl + g*Hg ...) -> dst [planes, G, P, Hg, R, D] at (g, r)
      "stats": src [H, n, T] (heads p*Hl ...)                  -> dst [Hl, P * n, T] at column r * n (global tile order)
      "out":   src [G, P, Hg, R, D] at (g, p)                  -> dst [H, R, D] at heads r*Hl + g*Hg ...
    """
    P, H, G, R, D, es = dims["P"], dims["H"], dims["G"], dims["R"], dims["D"], dims["es"]
    Hl = H // P
    Hg = Hl // G
    if kind == "qkv":
        plane = Hg * R * D * es
        return ((p * Hl + g * Hg) * R * D * es, H * R * D * es, (g * P + r) * plane, G * P * plane, plane,
                dims["planes"])
    if kind == "stats":
        n, T = dims["n"], dims["T"]
        w = n * T * es
        return p * Hl * w, w, r * w, P * w, w, Hl
    if kind == "out":
        w = Hg * R * D * es
        return (g * P + p) * w, w, (r * Hl + g * Hg) * R * D * es, w, w, 1
    raise ValueError(kind)
