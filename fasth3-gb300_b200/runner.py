"""H3FastRunner: the quantized DiT block loop on the h3b kernels, with sequence parallelism.

The reference's runner (fastvideo/models/dits/h3fast/__init__.py:406-553) permutes the packed tokens into compact
tile order, runs ``resid_norm_quant`` once, then per block: q/k/v GEMMs, ``qkv_prologue8``, tile scores, ``topk_rows``,
the FP8 VSA kernel, ``attn_gate_quant``, the out-projection, ``resid_norm_quant`` (gated residual + norm2 + modulate
+ quant), fc_in, the activation quantizer, fc_out and the next block's ``resid_norm_quant``. This runner keeps that
order and the buffers-owned-by-a-layout design, for BASELINE's architecture (which adds cross-attention to text and
uses GELU-tanh), and differs where the B200 kernels allow more fusion:

* the gated residuals (out-projection, cross-attention output, fc_out) and GELU-tanh are GEMM epilogues
  (``x <- x + gate * (row_scale * col_scale * acc)``), so no bf16 ``y`` round trip;
* q/k/v are one GEMM over the block's row-packed q/k/v weights (per-column global scales);
* Q/K E4M3 scales are per (head, tile) like V's (no per-layer static scales from the norm weights);
* the token dimension is sharded over ranks by whole tiles (``sp.SeqParallel``); the E4M3 Q/K/V tiles and the tile
  statistics cross ranks in one head all-to-all before attention and the bf16 attention output in one after
  (Ulysses-style, the exchange FastVideo's stock SP path makes, patches/fastvideo-a01c50a.patch:12-13). The reference
  runner itself is single-GPU (patch:644-645).

Every GEMM, norm, quantizer, prologue, selection and attention step is an h3b kernel; torch supplies the buffers,
the all-to-all (NCCL), the timestep MLP and the token permutation.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import ops
from .layout import (TILE, TileLayout, balanced_order, compute_topk, rope_3d, rope_positions, tile_layout,
                     tile_layout_from_metadata)
from .model import DiTModel, QuantLinear
from .reduction import TokenReduction, pair_maps
from .sp import PeerArena, SeqParallel, peer_copy_plan

LOG2E = 1.4426950408889634


@dataclass
class VsaMeta:
    """The VSA metadata the runner needs: the fields the reference reads from FastVideo's
    VideoSparseAttentionMetadata (__init__.py:171, 187-204, 440-445, 501-503) plus this runner's defaults.

    * ``grid``: the video latent (T, H, W); with no ``untile_combined_index`` the layout is built from it, the whole
      sequence is video and every query tile keeps ``topk`` key tiles.
    * ``untile_combined_index`` [S] / ``variable_block_sizes`` [n_tiles]: FastVideo's token -> slot map and tile
      sizes; the layout is then built from them (``layout.tile_layout_from_metadata``), prefix tiles first.
    * ``num_prefix_tiles``: exempt tiles (text, audio, references) every query tile attends to; their query tiles
      attend to every key tile.
    * ``video_tile_spans`` [(start, end)] with ``span_sparsities``: per span, compute_topk(sparsity, end - start) key
      tiles per query tile (the reference's sparse_ks); ``dense_layers``: blocks whose query tiles keep every tile of
      every span (dense_ks).
    * ``dense_prefix``: the reference's FASTVIDEO_H3_DENSE_PREFIX (one rank): the prefix queries against every key,
      and the other queries against the prefix keys, run as a separate dense pass (here this library's attention
      kernel with every such tile selected), and the sparse pass keeps the span tiles only; the gate quantizer merges
      the two by log-sum-exp (h3fast.cu:689-719)."""
    grid: tuple[int, int, int] | None = None
    topk: int = 32
    tile_elems: int = 64
    exempt: bool = True
    pad_tokens: int = 0
    untile_combined_index: torch.Tensor | None = None
    variable_block_sizes: torch.Tensor | None = None
    num_prefix_tiles: int = 0
    video_tile_spans: list | None = None
    span_sparsities: list | None = None
    dense_layers: tuple = ()
    dense_prefix: bool = False

    def selection(self, n_tiles: int, block: int) -> dict:
        """topk_rows' arguments for one block (the reference's _attn_cfg, __init__.py:440-445, and the dense-layer
        switch at :501-503)."""
        if self.video_tile_spans is None:
            if self.num_prefix_tiles:
                raise ValueError("num_prefix_tiles needs video_tile_spans")
            k = min(self.topk, n_tiles)
            return {"prefix": 0, "starts": [0], "ends": [n_tiles], "ks": [k], "split": False}
        spans = [(int(a), int(b)) for a, b in self.video_tile_spans]
        sparsities = self.span_sparsities if self.span_sparsities is not None else [None] * len(spans)
        if len(sparsities) != len(spans):
            raise ValueError("one sparsity per video tile span")
        if block in tuple(self.dense_layers):
            ks = [b - a for a, b in spans]
        else:
            ks = [min(self.topk, b - a) if sp is None else compute_topk(sp, b - a) for (a, b), sp in zip(spans, sparsities)]
        return {"prefix": int(self.num_prefix_tiles), "starts": [a for a, _ in spans], "ends": [b for _, b in spans],
                "ks": ks, "split": bool(self.dense_prefix and self.num_prefix_tiles > 0)}


class VirtualSeqParallel:
    """``world`` ranks run in one process, one after another per stage, on one GPU: the sharded block's data flow and
    exchange layouts without a second GPU (tests, and to check that the sharded result equals the single-rank one)."""

    def __init__(self, world: int):
        self.world = world

    def tiles(self, n_tiles: int, rank: int) -> tuple[int, int]:
        if n_tiles % (2 * self.world):
            raise ValueError(f"{n_tiles} tiles do not split into an even count per rank over {self.world} ranks")
        per = n_tiles // self.world
        return rank * per, (rank + 1) * per


class _Exchange:
    """The list-of-ranks form of the head all-to-all: one entry per rank this process hosts."""

    def __init__(self, sp):
        self.sp = sp
        self.world = sp.world
        self.virtual = isinstance(sp, VirtualSeqParallel)
        self.ranks = list(range(sp.world)) if self.virtual else [sp.rank]
        # when a list: (name, start event, end event) of every NCCL exchange is appended to it (device timing of the
        # collectives, read after the step; recording events does not synchronize)
        self.timing = None

    def _a2a(self, name: str, out: torch.Tensor, x: torch.Tensor) -> None:
        if self.timing is None:
            dist.all_to_all_single(out, x, group=self.sp.group)
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dist.all_to_all_single(out, x, group=self.sp.group)
        e1.record()
        self.timing.append((name, e0, e1))

    def tiles(self, n_tiles: int, rank: int) -> tuple[int, int]:
        return self.sp.tiles(n_tiles, rank) if self.virtual else self.sp.tiles(n_tiles)

    def seq_to_heads(self, xs: list[torch.Tensor], outs: list[torch.Tensor], name: str = "seq_to_heads") -> None:
        """[H, R, ...] per rank -> [P, Hl, R, ...] per rank, written into ``outs``."""
        P = self.world
        if not self.virtual:
            if P == 1:
                outs[0].copy_(xs[0].view(outs[0].shape)) if outs[0].data_ptr() != xs[0].data_ptr() else None
                return
            self._a2a(name, outs[0], xs[0])
            return
        Hl = xs[0].shape[0] // P
        for r in range(P):
            for p in range(P):
                outs[r][p].copy_(xs[p][r * Hl:(r + 1) * Hl])

    def heads_to_seq(self, ys: list[torch.Tensor], outs: list[torch.Tensor], name: str = "heads_to_seq") -> None:
        """[P, Hl, R, ...] per rank -> [H, R, ...] per rank."""
        P = self.world
        if not self.virtual:
            if P == 1:
                if outs[0].data_ptr() != ys[0].data_ptr():
                    outs[0].copy_(ys[0].view(outs[0].shape))
                return
            self._a2a(name, outs[0], ys[0])
            return
        Hl = ys[0].shape[1]
        for r in range(P):
            for p in range(P):
                outs[r][p * Hl:(p + 1) * Hl].copy_(ys[p][r])

    def heads_exchange(self, xs: list[torch.Tensor], outs: list[torch.Tensor], name: str = "qkv_e4m3") -> None:
        """One plane of Q, K or V: [H, R, D] per rank -> [G, P, Hg, R, D] per rank (head group g, source rank p: heads
        p*Hl + g*Hg .. of rank p's rows). Over NCCL G is 1 ([1, P, Hl, R, D] is the all-to-all's [P, Hl, R, D])."""
        P = self.world
        G = outs[0].shape[0]
        if not self.virtual:
            if P == 1:
                if outs[0].data_ptr() != xs[0].data_ptr():
                    outs[0].view(xs[0].shape).copy_(xs[0])
                return
            if G != 1:
                raise ValueError("the NCCL exchange sends all heads at once (one head group)")
            self._a2a(name, outs[0][0], xs[0])
            return
        Hl = xs[0].shape[0] // P
        Hg = Hl // G
        for r in range(P):
            for g in range(G):
                for p in range(P):
                    outs[r][g, p].copy_(xs[p][r * Hl + g * Hg:r * Hl + (g + 1) * Hg])

    def heads_return(self, ys: list[torch.Tensor], outs: list[torch.Tensor], name: str = "attn_out_bf16") -> None:
        """The attention output: [G, P, Hg, R, D] per rank -> [H, R, D] per rank (heads-first order)."""
        P = self.world
        G = ys[0].shape[0]
        if not self.virtual:
            if P == 1:
                if outs[0].data_ptr() != ys[0].data_ptr():
                    outs[0].copy_(ys[0].view(outs[0].shape))
                return
            if G != 1:
                raise ValueError("the NCCL exchange sends all heads at once (one head group)")
            self._a2a(name, outs[0], ys[0][0])
            return
        Hg = ys[0].shape[2]
        Hl = G * Hg
        for r in range(P):
            for g in range(G):
                for p in range(P):
                    outs[r][p * Hl + g * Hg:p * Hl + (g + 1) * Hg].copy_(ys[p][g, r])

    def all_gather_rows(self, xs: list[torch.Tensor], rows: list[int]) -> torch.Tensor:
        """Concatenation over ranks (in rank order) of each rank's [rows_r, C] block; ``rows`` holds every rank's
        row count."""
        if self.virtual:
            return torch.cat([x[:r] for x, r in zip(xs, rows)])
        if self.world == 1:
            return xs[0][:rows[0]]
        m = max(rows)
        x = xs[0]
        buf = torch.empty(m, x.shape[1], device=x.device, dtype=x.dtype)
        buf[:x.shape[0]].copy_(x)
        out = torch.empty(self.world * m, x.shape[1], device=x.device, dtype=x.dtype)
        dist.all_gather_into_tensor(out, buf, group=self.sp.group)
        return torch.cat([out[p * m:p * m + rows[p]] for p in range(self.world)])


@dataclass
class _RankState:
    """One rank's shard layout and buffers (the reference's _Layout.buffers, __init__.py:207-252)."""
    rank: int
    lay: TileLayout        # this rank's tiles, rows renumbered from 0
    first: int
    rows: int
    rows_pad: int
    n_local: int
    tok_index: torch.Tensor  # int64 [rows] global token of each local row
    b: dict = field(default_factory=dict)
    arena: PeerArena | None = None  # the receive buffers and flags of the peer transport


def _fused_rows(lins: list[QuantLinear]) -> dict:
    """The packed operand of several row-packed linears as one GEMM B operand, plus per-column global scales."""
    fmt = lins[0].fmt
    if fmt == "nvfp4":
        ws = [lin._nvfp4_weight for lin in lins]
        sfs = [lin._nvfp4_weight_scale for lin in lins]
    else:
        ws = [lin._fp8_weight for lin in lins]
        sfs = None
    adjacent = all(ws[i + 1].data_ptr() == ws[i].data_ptr() + ws[i].numel() * ws[i].element_size()
                   for i in range(len(ws) - 1)) and all(w.is_contiguous() for w in ws)
    N = sum(w.shape[0] for w in ws)
    if adjacent:
        w = ws[0].as_strided((N, ws[0].shape[1]), ws[0].stride())
        sf = None if sfs is None else sfs[0].as_strided((N, sfs[0].shape[1]), sfs[0].stride())
    else:
        w = torch.cat(ws)
        sf = None if sfs is None else torch.cat(sfs)
    if fmt == "nvfp4":
        col = torch.cat([lin._nvfp4_alpha.float().reshape(1).expand(lin.out_features) for lin in lins]).contiguous()
    else:
        col = torch.cat([lin._fp8_weight_scale.float().reshape(-1).expand(lin.out_features) for lin in lins])
    return {"w": w, "sf": sf, "col": col.contiguous(), "fmt": fmt, "N": N}


class H3FastRunner:
    """All blocks of a DiTModel on the h3b kernels. ``sp``: a SeqParallel (one rank per process; NCCL on GPUs), a
    VirtualSeqParallel (all ranks in this process), or None (this GPU alone, even inside an initialized process
    group). ``qk_int8``: the self-attention's Q and K as per-tile int8 with the QK^T on the tensor cores' integer path
    (exact scores; E4M3 otherwise). ``v_f16``: V tiles as f16 (see below)."""

    def __init__(self, model: DiTModel, sp: SeqParallel | VirtualSeqParallel | None = None, qk_int8: bool = False,
                 v_f16: bool = False, ffn_requant: str = "rows", exchange: str = "auto", head_groups: int | None = None,
                 attn_kernel: str = "wide", tile_order: str = "reference"):
        self.model = model
        self.qk_int8 = bool(qk_int8)
        # FFN re-quantization between fc_in and fc_out: "rows" -- the reference's rule, the bf16 fc_in output
        # re-quantized per row (global scale amax_row / 2688) by a separate pass; "static" -- fc_in's epilogue writes
        # NVFP4 directly under a fixed global scale per block, s_i = headroom * max|u_i| / 2688 recorded by the first
        # forward (which runs the "rows" path; max over ranks) and kept; values above headroom x that maximum saturate
        if ffn_requant not in ("rows", "static"):
            raise ValueError(f"ffn_requant must be 'rows' or 'static', not {ffn_requant!r}")
        self.ffn_requant = ffn_requant
        self.ffn_headroom = 2.0
        # self-attention kernel: "wide" (h3b_vsa_fp8_ws: one weight-stationary M=64 MMA advances both key streams of
        # a query tile; needs f16 V and E4M3 Q/K) or "tile" (h3b_vsa_fp8_ex: two M=64 streams, E4M3 or f16 V, int8
        # Q/K). The two give the same output.
        if attn_kernel not in ("wide", "tile"):
            raise ValueError(f"attn_kernel must be 'wide' or 'tile', not {attn_kernel!r}")
        self.attn_kernel = "tile" if self.qk_int8 else attn_kernel
        # tile order of a layout built from meta.grid: "reference" -- (t, h, w), the reference runner's; "balanced" --
        # layout.balanced_order, the edge cubes' smaller tiles spread evenly so every rank's contiguous shard holds its
        # share of rows (per token the same attention up to the order of each query tile's selected key tiles; a
        # forward's result is the same at every rank count for either order)
        if tile_order not in ("reference", "balanced"):
            raise ValueError(f"tile_order must be 'reference' or 'balanced', not {tile_order!r}")
        self.tile_order = tile_order
        # self-attention V tiles as f16 holding the E4M3 values (decoded once by the prologue, loaded by the PV MMAs as
        # is; the wide kernel's form), or, with the tile kernel, as E4M3 codes converted by the attention kernel on
        # every use (half the bytes in the prologue's writes and the exchange); the results are bit-identical. The
        # cross-attention's text V is always f16.
        self.v_dtype = torch.float16 if (v_f16 or self.attn_kernel == "wide") else torch.uint8
        self.blocks = list(model.transformer_blocks)
        cfg = model.config
        self.cfg = cfg
        self.heads, self.head_dim, self.hidden, self.ffn = cfg.heads, cfg.head_dim, cfg.hidden, cfg.ffn
        if self.head_dim != 128:
            raise ValueError("head_dim 128 only")
        self.fp4 = cfg.fmt == "nvfp4"
        if ffn_requant == "static" and not self.fp4:
            raise ValueError("ffn_requant='static' needs NVFP4 linears")
        self.ex = _Exchange(sp if sp is not None else SeqParallel.local())
        if self.heads % self.ex.world:
            raise ValueError(f"{self.heads} heads do not split over {self.ex.world} ranks")
        self.layouts: dict[tuple, list[_RankState]] = {}
        self.refresh_weights()
        dev = self.blocks[0].scale_shift_table.device
        self.dev = dev
        self.ones_c = torch.ones(self.hidden, device=dev, dtype=torch.bfloat16)
        self.ffn_scales = torch.zeros(len(self.blocks), device=dev)  # "static": s_i once recorded
        self._ffn_amax = torch.zeros(len(self.blocks), device=dev)
        self._ffn_state = "unset"  # "unset" -> "recording" (during the first forward) -> "set"
        self.text_cache: dict = {}
        # the gate-compress branch (gate GEMM, compressed attention) runs on this stream beside the sparse attention
        # (the reference's side stream, __init__.py:465-535)
        self.side = torch.cuda.Stream(dev) if any(f["gate"] is not None for f in self.fused) else None
        # trace(block, stage, rank, {name: tensor}) after each stage when set (tests and debugging); the tensors are the
        # live buffers, so a tracer that keeps them must copy them
        self.trace = None
        # read the kernels' device status words after each forward's last kernel and raise on a failure (a bounded
        # wait that expired, a selection list longer than the attention kernel holds); costs one host sync per step
        self.check_status = True
        # the head exchange's transport: "local" (one rank), "virtual" (emulated ranks), "nccl" (all_to_all_single),
        # or "peer" (copy engines into peer-mapped receive buffers with flag words, sp.PeerArena); "auto" takes
        # "peer" when every rank can map every other rank's memory, else NCCL
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError(f"exchange must be 'auto', 'peer' or 'nccl', not {exchange!r}")
        P = self.ex.world
        self.transport_note = None
        if P == 1:
            self.transport = "local"
        elif self.ex.virtual:
            self.transport = "virtual"
        elif exchange == "nccl":
            self.transport = "nccl"
        else:
            why = self._peer_probe()
            if why is not None and exchange == "peer":
                raise RuntimeError(f"peer exchange unavailable: {why}")
            self.transport, self.transport_note = ("peer", None) if why is None else ("nccl", why)
        # head groups of the attention pipeline: with the peer transport, group g's attention runs while later groups'
        # Q/K/V are still arriving and earlier groups' outputs are on their way back (the virtual transport uses the
        # same layout, so one GPU tests it); NCCL and one rank take all heads at once
        Hl = self.heads // P
        if head_groups is None:
            G = 1 if self.transport in ("local", "nccl") else \
                next(d for d in range(min(4, Hl), Hl + 1) if Hl % d == 0)
        else:
            G = int(head_groups)
            if G < 1 or Hl % G or (G > 1 and self.transport in ("local", "nccl")):
                raise ValueError(f"head_groups={G}: must divide the {Hl} heads per rank; more than one group needs "
                                 f"the peer or virtual transport")
        self.head_groups = G
        # peer transport: send the tile statistics (about 1 MB per receiver at 8 ranks) with one SM kernel
        # (h3b_peer_put) instead of five copies and a flag write per receiver on the copy engines. Off by default: on
        # 2 GPUs it left the wait for the statistics unchanged (the wait there is skew between the ranks, not copy
        # latency), and the copy-engine form is the one measured on 8
        self.stats_put = False
        self._epoch = 0  # exchanges so far (the peer transport's flag value), the same count on every rank
        self._copy_streams: list | None = None

    def _peer_probe(self) -> str | None:
        """Maps a small arena over the ranks and releases it (collective): None when every rank can map every other
        rank's memory, else why not."""
        try:
            ar = PeerArena(self.ex.sp, self.dev, {"probe": ((4096,), torch.uint8)}, 1)
        except RuntimeError as exc:
            return str(exc)
        ar.close(self.ex.sp.group)
        return None

    def close(self) -> None:
        """Releases the peer arenas of every layout (collective over the ranks when the transport is "peer")."""
        for _, states in self.layouts.values():
            for st in states:
                if st.arena is not None:
                    st.arena.close(self.ex.sp.group)
                    st.arena = None
        self.layouts.clear()

    def refresh_weights(self) -> None:
        """(Re)builds the GEMM B operands of every block from its linears' packed weights: at construction, and after
        a linear's weights were replaced (a LoRA adapter merged or removed, ``weights.merge_lora_into``). The cached
        text keys/values are dropped with them."""
        self.fused = []
        for blk in self.blocks:
            a, c = blk.attn, blk.attn2
            self.fused.append({
                "qkv": _fused_rows([a.to_q, a.to_k, a.to_v]), "o": _fused_rows([a.to_out]),
                "cq": _fused_rows([c.to_q]), "ckv": _fused_rows([c.to_k, c.to_v]), "co": _fused_rows([c.to_out]),
                "fc_in": _fused_rows([blk.ff.fc_in]), "fc_out": _fused_rows([blk.ff.fc_out]),
                "gate": _fused_rows([a.to_gate_compress]) if a.to_gate_compress is not None else None})
        if hasattr(self, "text_cache"):
            self.text_cache.clear()

    @staticmethod
    def supported(model: DiTModel, meta: VsaMeta) -> bool:
        """The reference's gate (__init__.py:164-171): packed FP8 or NVFP4 linears, exempt metadata, 64-token tiles."""
        blk = model.transformer_blocks[0]
        lins = (blk.attn.to_q, blk.attn.to_k, blk.attn.to_v, blk.attn.to_out, blk.ff.fc_in, blk.ff.fc_out)
        fp4 = all(getattr(lin, "_nvfp4_weight", None) is not None for lin in lins)
        fp8 = all(getattr(lin, "_fp8_weight", None) is not None for lin in lins)
        return (fp4 or fp8) and meta is not None and meta.exempt and not meta.pad_tokens and meta.tile_elems == 64

    # ------------------------------------------------------------------------------------------------- GEMM
    def _gemm(self, a, a_sf, fused, out, *, row_scale=None, act=None, residual=None, gate=None, cols=None,
              alpha_dev=None):
        w, sf, col = fused["w"], fused["sf"], fused["col"]
        if cols is not None:
            w, col = w[cols], col[cols]
            sf = None if sf is None else sf[cols]
        if fused["fmt"] == "nvfp4":
            ops.gemm_nvfp4(a, a_sf, w, sf, out, scale_a=row_scale, scale_b=col, act=act, residual=residual,
                           gate=gate, alpha_dev=alpha_dev)
        else:
            ops.gemm_fp8(a, w, out, scale_a=row_scale, scale_b=col, act=act, residual=residual, gate=gate,
                         alpha_dev=alpha_dev)

    def reset_ffn_scales(self) -> None:
        """With ffn_requant="static": the next forward records the FFN global scales again (e.g. after new
        weights)."""
        self._ffn_state = "unset"

    # ------------------------------------------------------------------------------------------------- layout
    def _layouts(self, meta: VsaMeta, rotary, tag: object = None) -> tuple[TileLayout, list[_RankState]]:
        by_meta = meta.untile_combined_index is not None
        src = (meta.untile_combined_index.data_ptr(), meta.untile_combined_index.numel()) if by_meta else \
            tuple(meta.grid)
        key = (src, self.ex.world, tuple(self.ex.ranks), tag, None if rotary is None else rotary[0].data_ptr())
        hit = self.layouts.get(key)
        if hit is not None:
            return hit
        P = self.ex.world
        if by_meta:
            if meta.variable_block_sizes is None:
                raise ValueError("untile_combined_index needs variable_block_sizes")
            full = tile_layout_from_metadata(meta.untile_combined_index, meta.variable_block_sizes, pad_to=2 * P)
        else:
            full = tile_layout(*meta.grid, pad_to=2 * P)
        if self.tile_order == "balanced":
            if by_meta:
                raise ValueError("tile_order='balanced' needs a layout from meta.grid (metadata layouts keep their "
                                 "prefix tiles first)")
            full = balanced_order(full)
        if full.n_ext != full.n_tiles:
            raise ValueError(f"{full.n_tiles} tiles do not split into an even count per rank over {P} ranks")
        if rotary is None:
            if full.grid is None:
                raise ValueError("a layout from metadata needs the rotary tables (cos, sin) of its tokens")
            cos, sin = rope_3d(full)
        else:
            cos, sin = (t.reshape(-1, t.shape[-1])[full.perm] for t in rotary)
        H, D, C, F = self.heads, self.head_dim, self.hidden, self.ffn
        Hl = H // P
        n_all = full.n_tiles
        dev = self.dev
        u8, bf, f32, i32 = torch.uint8, torch.bfloat16, torch.float32, torch.int32
        states = []
        for r in self.ex.ranks:
            first, last = self.ex.tiles(n_all, r)
            lay = full.shard(first, last)
            R, n_local = lay.rows, lay.n_ext
            rows_pad = n_local * TILE
            r0 = int(full.tile_row0[first])
            st = _RankState(r, lay, first, R, rows_pad, n_local, full.perm[r0:r0 + R].to(dev))
            hb = C // 2 if self.fp4 else C
            fb = F // 2 if self.fp4 else F
            b = st.b
            b["tile_row0"], b["vbs"] = lay.tile_row0.to(dev), lay.vbs.to(dev)
            b["slot"] = lay.slot.to(dev)
            b["cos"], b["sin"] = cos[r0:r0 + R].contiguous().to(dev), sin[r0:r0 + R].contiguous().to(dev)
            b["x"] = torch.empty(R, C, device=dev, dtype=bf)
            b["h"] = torch.empty(R, hb, device=dev, dtype=u8)
            b["h_sf"] = torch.zeros(ops.sf_rows(R), C // 16, device=dev, dtype=u8) if self.fp4 else None
            b["hs"] = torch.empty(R, device=dev, dtype=f32)
            b["qkv"] = torch.empty(R, 3 * C, device=dev, dtype=bf)
            # E4M3 (or int8) Q, K and V planes [H, rows_pad, 128] of this rank's rows; Q/K (and an E4M3 V) are planes
            # of one tensor so one 2D copy sends all of a head group's planes. Head-sharded side: [G, P, Hg, rows_pad,
            # 128] per plane -- head group g, chunk p = rank p's rows (what the attention kernel reads with chunks=P)
            G = self.head_groups
            Hg = Hl // G
            planes = 3 if self.v_dtype == u8 else 2
            peer = self.transport == "peer"
            stat_names = [("qs", ()), ("ks", ()), ("vs", ()), ("qp", (D,)), ("kp", (D,))]
            if self.side is not None:
                stat_names.append(("vp", (D,)))
            b["qkv_s"] = torch.zeros(planes, H, rows_pad, D, device=dev, dtype=u8)
            b["qb"], b["kb"] = b["qkv_s"][0], b["qkv_s"][1]
            b["vb"] = b["qkv_s"][2] if planes == 3 else torch.zeros(H, rows_pad, D, device=dev, dtype=self.v_dtype)
            if peer:  # every receive buffer in one allocation that the other ranks map
                regions = {"qkv_x": ((planes, G, P, Hg, rows_pad, D), u8)}
                if planes == 2:
                    regions["v_x"] = ((G, P, Hg, rows_pad, D), self.v_dtype)
                for nm, tail in stat_names:
                    regions[nm + "_all"] = ((Hl, n_all, *tail), f32)
                regions["ob"] = ((H, rows_pad, D), bf)
                st.arena = PeerArena(self.ex.sp, dev, regions, 1 + 2 * G)
                rx = st.arena.tensors
            else:
                rx = {}
            if P == 1:
                b["qkv_x"] = b["qkv_s"].view(planes, 1, 1, H, rows_pad, D)
                v_x = b["vb"].view(1, 1, H, rows_pad, D)
            else:
                b["qkv_x"] = rx["qkv_x"] if peer else torch.zeros(planes, G, P, Hg, rows_pad, D, device=dev, dtype=u8)
                v_x = None if planes == 3 else (rx["v_x"] if peer else
                                                torch.zeros(G, P, Hg, rows_pad, D, device=dev, dtype=self.v_dtype))
            b["qb_x"], b["kb_x"] = b["qkv_x"][0], b["qkv_x"][1]
            b["vb_x"] = b["qkv_x"][2] if planes == 3 else v_x
            # per (head, tile) E4M3 scales and tile means, local tiles; their exchange buffers; all tiles
            for nm, tail in stat_names:
                b[nm] = torch.zeros(H, n_local, *tail, device=dev, dtype=f32)
                if P == 1:
                    b[nm + "_x"] = b[nm].view(1, H, n_local, *tail)
                    b[nm + "_all"] = b[nm]
                elif peer:  # written in global tile order by the senders' copies
                    b[nm + "_all"] = rx[nm + "_all"]
                else:
                    b[nm + "_x"] = torch.zeros(P, Hl, n_local, *tail, device=dev, dtype=f32)
                    b[nm + "_all"] = torch.zeros(Hl, n_all, *tail, device=dev, dtype=f32)
            if self.side is None:
                b["vp"] = torch.empty(H, n_local, D, device=dev, dtype=f32)
            else:  # gate-compress branch
                b["g"] = torch.empty(R, C, device=dev, dtype=bf)
                b["oc"] = torch.zeros(H, n_local, D, device=dev, dtype=bf)
                if P > 1:
                    b["oc_all"] = torch.zeros(Hl, n_all, D, device=dev, dtype=bf)
                    b["oc_x"] = torch.zeros(P, Hl, n_local, D, device=dev, dtype=bf)
                else:
                    b["oc_all"], b["oc_x"] = b["oc"], b["oc"].view(1, H, n_local, D)
            b["vs_head"] = torch.empty(Hl, device=dev, dtype=f32)
            b["sc"] = torch.empty(Hl, n_all, n_all, device=dev, dtype=f32)
            b["idx"] = torch.empty(Hl, n_all, n_all, device=dev, dtype=i32)
            b["num"] = torch.zeros(Hl, n_all, device=dev, dtype=i32)
            b["vbs_all"] = full.vbs.to(dev)
            b["ob"] = rx["ob"] if peer else torch.zeros(H, rows_pad, D, device=dev, dtype=bf)
            b["ob_x"] = torch.zeros(G, P, Hg, rows_pad, D, device=dev, dtype=bf) if P > 1 else \
                b["ob"].view(1, 1, H, rows_pad, D)
            b["a"] = torch.empty(R, hb, device=dev, dtype=u8)
            b["a_sf"] = torch.zeros(ops.sf_rows(R), C // 16, device=dev, dtype=u8) if self.fp4 else None
            b["as"] = torch.empty(R, device=dev, dtype=f32)
            # cross-attention: queries of this rank's rows, every head; all text tiles selected
            b["cq"] = torch.empty(R, C, device=dev, dtype=bf)
            b["cqb"] = torch.zeros(H, rows_pad, D, device=dev, dtype=u8)
            b["cqs"] = torch.zeros(H, n_local, device=dev, dtype=f32)
            b["cob"] = torch.zeros(H, rows_pad, D, device=dev, dtype=bf)
            n_txt = self.cfg.text_len // TILE
            b["cidx"] = torch.arange(n_txt, device=dev, dtype=i32).repeat(H, n_local, 1).contiguous()
            b["cnum"] = torch.full((H, n_local), n_txt, device=dev, dtype=i32)
            b["u"] = torch.empty(R, F, device=dev, dtype=bf)
            b["f"] = torch.empty(R, fb, device=dev, dtype=u8)
            b["f_sf"] = torch.zeros(ops.sf_rows(R), F // 16, device=dev, dtype=u8) if self.fp4 else None
            b["fs"] = torch.empty(R, device=dev, dtype=f32)
            states.append(st)
        self.layouts[key] = (full, states)
        return full, states

    # ------------------------------------------------------------------------------------------------- text K/V
    def _text_kv(self, context: torch.Tensor) -> dict:
        """Per block: E4M3 text keys (RMSNorm) and values [H, L, 128] with per-(head, tile) scales; cached for the
        last context tensor (the text embedding is fixed over the denoising steps)."""
        key = (context.data_ptr(), context._version, tuple(context.shape))
        if self.text_cache.get("key") == key:
            return self.text_cache
        cfg = self.cfg
        L = context.shape[-2]
        if L % TILE:
            raise ValueError("text length must be a multiple of 64")
        ctx = context.reshape(L, -1).contiguous()
        H, D, C, dev = self.heads, self.head_dim, self.hidden, self.dev
        n_txt = L // TILE
        tq = torch.empty(L, ctx.shape[1] // 2 if self.fp4 else ctx.shape[1], device=dev, dtype=torch.uint8)
        tsf = torch.zeros(ops.sf_rows(L), ctx.shape[1] // 16, device=dev, dtype=torch.uint8) if self.fp4 else None
        ts = torch.empty(L, device=dev, dtype=torch.float32)
        if self.fp4:
            ops.quant_nvfp4_rows(ctx, tq, tsf, ts)
        else:
            ops.quant_fp8_rows(ctx, tq.view(ops.FP8), ts)
        kv = torch.empty(L, 2 * C, device=dev, dtype=torch.bfloat16)
        row0 = torch.arange(n_txt, device=dev, dtype=torch.int32) * TILE
        vbs = torch.full((n_txt,), TILE, device=dev, dtype=torch.int32)
        kb = torch.zeros(len(self.blocks), H, L, D, device=dev, dtype=torch.uint8)
        # text V always as f16 holding the E4M3 values (bit-identical results; a few MB per block, and the
        # cross-attention's PV MMAs load it as is instead of converting every use)
        vb = torch.zeros(len(self.blocks), H, L, D, device=dev, dtype=torch.float16)
        ks = torch.zeros(len(self.blocks), H, n_txt, device=dev, dtype=torch.float32)
        vs = torch.zeros_like(ks)
        vs_head = torch.zeros(len(self.blocks), H, device=dev, dtype=torch.float32)
        for i, blk in enumerate(self.blocks):
            self._gemm(tq if self.fp4 else tq.view(ops.FP8), tsf, self.fused[i]["ckv"], kv)
            ops.head_tile_quant(kv[:, :C], ts, row0, vbs, blk.attn2.norm_k.weight, kb[i], ks[i], None, H, n_txt,
                                blk.attn2.norm_k.eps)
            ops.head_tile_quant(kv[:, C:], ts, row0, vbs, None, vb[i], vs[i], vs_head[i], H, n_txt)
            if self.trace is not None:
                self.trace(i, "text", self.ex.ranks[0], {"tq": tq, "tsf": tsf, "ts": ts, "kv": kv, "kb": kb[i],
                                                          "vb": vb[i], "ks": ks[i], "vs": vs[i]})
        self.text_cache = {"key": key, "kb": kb, "vb": vb, "ks": ks, "vs": vs, "vs_head": vs_head, "n": n_txt,
                           "vbs": vbs, "L": L}
        return self.text_cache

    # ------------------------------------------------------------------------------------------------- forward
    def forward(self, packed: torch.Tensor, temb: torch.Tensor, adaln_indices: torch.Tensor | None,
                rotary: tuple[torch.Tensor, torch.Tensor] | None, meta: VsaMeta,
                context: torch.Tensor | None = None, reduction: TokenReduction | None = None) -> torch.Tensor:
        """All blocks; ``packed`` [1, S, C] bf16 in token order (the full sequence on every rank), ``temb`` [1, C]
        timestep embedding, ``adaln_indices`` [S] int (table row per token; None: one row), ``rotary`` (cos, sin)
        [S, 96] in token order (None: 3D RoPE from meta.grid), ``context`` [1, L, 4096] text. Returns [1, S, C] in
        token order, identical on every rank (the shards are gathered at the end). ``reduction`` (one rank only, like
        the reference runner): blocks [begin, end) run on horizontally paired tokens (``reduction.build_token_reduction``
        over meta.grid), pooled before block ``begin`` and expanded before block ``end`` (__init__.py:406-430)."""
        if context is None:
            raise ValueError("the cross-attention needs context")
        full, states = self._layouts(meta, rotary)
        S = packed.shape[-2]
        if S != full.rows:
            raise ValueError(f"packed has {S} tokens, the layout has {full.rows}")
        if meta.dense_prefix and meta.num_prefix_tiles and self.ex.world != 1:
            raise ValueError("the dense-prefix pass runs on one rank (like the reference runner)")
        if temb.reshape(-1, self.hidden).shape[0] != 1:
            raise ValueError("one timestep per forward: the gates are GEMM-epilogue column vectors")
        if adaln_indices is not None and bool((adaln_indices != 0).any()):
            raise ValueError("adaln_indices must select table row 0 (one timestep)")
        tabs = self.model.adaln_tables(temb.reshape(1, -1))  # [blocks, 6, C]
        txt = self._text_kv(context)
        if self.ffn_requant == "static" and self._ffn_state == "unset":
            self._ffn_amax.zero_()
            self._ffn_state = "recording"
        x_in = packed.reshape(S, -1)
        for st in states:
            torch.index_select(x_in, 0, st.tok_index, out=st.b["x"])
            st.b["adaln"] = None
        for st in states:
            self._norm(st, self.blocks[0].eps, tabs[0, 0:1], tabs[0, 1:2], 0)
        red = self._reduced(reduction, meta) if reduction is not None else None
        cur = (full, states, meta)
        for i, blk in enumerate(self.blocks):
            if red is not None and i in (reduction.begin, reduction.end):
                L, Rst = states[0].b, red["states"][0].b
                if i == reduction.begin:
                    ops.pool_pairs(L["x"], red["ia"], red["ib"], Rst["x"], red["pooled"])
                    cur = (red["full"], red["states"], red["meta"])
                else:
                    ops.expand_pairs(L["x"], Rst["x"], red["pooled"], red["par"], red["pair"], reduction.update_scale)
                    cur = (full, states, meta)
                # the previous block ended with this block's norm1 on the other layout
                self._norm(cur[1][0], blk.eps, tabs[i, 0:1], tabs[i, 1:2], i)
            self._block(i, blk, cur[0], cur[1], tabs, txt, cur[2])
        if red is not None and reduction.begin < len(self.blocks) <= reduction.end:
            ops.expand_pairs(states[0].b["x"], red["states"][0].b["x"], red["pooled"], red["par"], red["pair"],
                             reduction.update_scale)
        if self._ffn_state == "recording":
            if not self.ex.virtual and self.ex.world > 1:
                dist.all_reduce(self._ffn_amax, op=dist.ReduceOp.MAX, group=self.ex.sp.group)
            torch.mul(self._ffn_amax, self.ffn_headroom / 2688.0, out=self.ffn_scales)
            self.ffn_scales.clamp_(min=1e-12)
            self._ffn_state = "set"
        per = full.n_tiles // self.ex.world
        rows_all = [int(full.vbs[p * per:(p + 1) * per].sum()) for p in range(self.ex.world)]
        out = self.ex.all_gather_rows([st.b["x"] for st in states], rows_all)  # global tile order
        inv = self.__dict__.setdefault("_inv_cache", {}).get(id(full))
        if inv is None or inv[0] is not full:
            t = torch.empty_like(full.perm)
            t[full.perm] = torch.arange(full.rows)
            inv = self._inv_cache[id(full)] = (full, t.to(out.device))
        result = out.index_select(0, inv[1]).unsqueeze(0)
        if self.check_status and not torch.cuda.is_current_stream_capturing():
            ops.check_status(self.dev)
        return result

    def _reduced(self, plan: TokenReduction, meta: VsaMeta) -> dict:
        """The paired layout of ``plan`` (its grid at half width, RoPE at the pairs' mean positions) and the compact-row
        maps between it and the full layout (``_pair_maps``, __init__.py:262-278), cached per plan."""
        if self.ex.world != 1:
            raise ValueError("token reduction runs on one rank (the reference runner is single-GPU)")
        if self.tile_order != "reference":
            raise ValueError("token reduction pairs tiles in the reference tile order")
        if tuple(plan.grid) != tuple(meta.grid) or plan.video_start != 0:
            raise ValueError(f"the reduction plan's grid {plan.grid} (video_start {plan.video_start}) is not "
                             f"the sequence's {tuple(meta.grid)}")
        cache = self.__dict__.setdefault("_red_cache", {})
        hit = cache.get(id(plan))
        if hit is not None and hit["plan"] is plan:
            return hit
        cache.clear()
        rmeta = dataclasses.replace(meta, grid=plan.reduced_grid)
        rotary = rope_positions(plan.positions)
        rfull, rstates = self._layouts(rmeta, rotary, tag=("pairs", plan.positions.data_ptr()))
        for st in rstates:
            st.b["adaln"] = None  # one timestep: every pair takes table row 0, as its first source does
        full, _ = self._layouts(meta, None)
        maps = pair_maps(plan, full.perm, rfull.perm)
        dev = self.dev
        hit = {"plan": plan, "meta": rmeta, "full": rfull, "states": rstates,
               "ia": maps["ia"].to(dev), "ib": maps["ib"].to(dev), "par": maps["par"].to(dev),
               "pair": maps["pair"].to(dev), "pooled": torch.empty(rfull.rows, self.hidden, device=dev,
                                                                    dtype=torch.bfloat16)}
        cache[id(plan)] = hit
        return hit

    def _norm(self, st: _RankState, eps: float, shift: torch.Tensor, scale: torch.Tensor, i: int,
              stage: str = "norm1") -> None:
        b = st.b
        ops.resid_norm_quant(b["x"], None, None, None, b["adaln"], None, shift, scale, b["x"], b["h"], b["h_sf"],
                             b["hs"], eps, norm="layer")
        self._t(i, stage, st, x=b["x"], h=b["h"], h_sf=b["h_sf"], hs=b["hs"])

    def _block(self, i: int, blk, full: TileLayout, states: list[_RankState], tabs: torch.Tensor, txt: dict,
               meta: VsaMeta) -> None:
        H, D, C = self.heads, self.head_dim, self.hidden
        P = self.ex.world
        Hl = H // P
        n_all = full.n_tiles
        fz = self.fused[i]
        tab = tabs[i]  # [6, C]: shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp
        sm_scale = 1.0 / math.sqrt(D)
        gate = fz["gate"] is not None
        main = torch.cuda.current_stream(self.dev)
        # ---- q/k/v GEMM (row scale deferred to the prologue) and the prologue, on each rank's rows
        for st in states:
            b = st.b
            if gate:  # g = h @ Wg^T on the side stream (h's row scale is applied by the gate quantizer, as sg)
                self.side.wait_stream(main)
                with torch.cuda.stream(self.side):
                    self._gemm(b["h"], b["h_sf"], fz["gate"], b["g"])
            self._gemm(b["h"], b["h_sf"], fz["qkv"], b["qkv"])
            self._t(i, "qkv", st, qkv=b["qkv"])
            self._prologue(st, blk)
            self._t(i, "prologue", st, qb=b["qb"], kb=b["kb"], vb=b["vb"], qs=b["qs"], ks=b["ks"], vs=b["vs"],
                    qp=b["qp"], kp=b["kp"])
        # ---- sequence -> heads
        G = self.head_groups
        Hg = Hl // G
        peer = self.transport == "peer"
        stats = ("qs", "ks", "vs", "qp", "kp") + (("vp",) if gate else ())
        if peer:
            self._epoch += 1
            self._peer_send_heads(states[0], stats)
        else:
            planes = [("qb", "qb_x"), ("kb", "kb_x"), ("vb", "vb_x")]
            for src, dst in planes:
                self.ex.heads_exchange([st.b[src] for st in states], [st.b[dst] for st in states], "qkv_e4m3")
            for nm in stats:
                self.ex.seq_to_heads([st.b[nm] for st in states], [st.b[nm + "_x"] for st in states], "tile_stats")
        # ---- coarse step and sparse attention over this rank's heads, every rank's rows
        for st in states:
            b = st.b
            if peer:
                self._peer_wait(st, 0, 1, "wait_tile_stats")
            elif P > 1:  # [P, Hl, n_local, ...] -> [Hl, n_all, ...] in global tile order
                for nm in stats:
                    src = b[nm + "_x"]
                    b[nm + "_all"].copy_(src.transpose(0, 1).reshape(b[nm + "_all"].shape))
            torch.amax(b["vs_all"], dim=1, out=b["vs_head"])
            ops.tile_scores(b["qp_all"], b["kp_all"], b["sc"], sm_scale)
            sel = meta.selection(n_all, i)
            ops.topk_rows(b["sc"], n_all, n_all, sel["prefix"], sel["starts"], sel["ends"], sel["ks"], b["idx"],
                          b["num"], sel["split"])
            if gate:  # compressed branch oc = softmax(sc) @ vp on the side stream, beside the sparse attention
                self.side.wait_stream(main)
                with torch.cuda.stream(self.side):
                    ops.compressed_branch(b["sc"], b["vp_all"], b["oc_all"])
            self._t(i, "select", st, qb_x=b["qb_x"], kb_x=b["kb_x"], vb_x=b["vb_x"], qs_all=b["qs_all"],
                    ks_all=b["ks_all"], vs_all=b["vs_all"], qp_all=b["qp_all"], kp_all=b["kp_all"],
                    vs_head=b["vs_head"], sc=b["sc"], idx=b["idx"], num=b["num"], vp_all=b.get("vp_all"))
            lse2 = self._buf(b, "lse2", (Hl, st.rows_pad), torch.float32) if sel["split"] else None
            for g in range(G):  # head group g: [P, Hg, rows_pad, 128] planes, heads g*Hg .. of this rank's
                hs = slice(g * Hg, (g + 1) * Hg)
                if peer:
                    self._peer_wait(st, 1 + g, 1, "wait_qkv")
                ops.vsa_fp8_ex(b["qb_x"][g], b["kb_x"][g], b["vb_x"][g], b["ob_x"][g], b["idx"][hs], b["num"][hs],
                               b["vbs_all"], b["vbs_all"], b["vs_all"][hs], b["vs_head"][hs], sm_scale * LOG2E, Hg,
                               n_all, n_all, st.rows_pad, st.rows_pad, chunks_q=P, chunks_kv=P, qs=b["qs_all"][hs],
                               ks=b["ks_all"][hs], lse=None if lse2 is None else lse2[hs], idx_ld=n_all,
                               q_scale_ld=n_all, kv_scale_ld=n_all, qk_int8=self.qk_int8,
                               wide=self.attn_kernel == "wide")
                if peer:
                    self._peer_send_out(st, g)
            if sel["split"]:
                self._dense_prefix(st, sel["prefix"], n_all, sm_scale)
                self._t(i, "dense_prefix", st, o1=b["o1"], lse1a=b["lse1a"], lse1b=b["lse1b"], lse2=b["lse2"],
                        ob_x=b["ob_x"])
            self._t(i, "attn", st, ob_x=b["ob_x"])
        # ---- heads -> sequence
        if peer:
            self._peer_wait(states[0], 1 + G, G, "wait_attn_out")
        else:
            self.ex.heads_return([st.b["ob_x"] for st in states], [st.b["ob"] for st in states], "attn_out_bf16")
        if gate:
            main.wait_stream(self.side)
            if P > 1:  # [Hl, n_all, D] -> [P, Hl, n_local, D] -> every head of this rank's tiles
                for st in states:
                    b = st.b
                    b["oc_x"].copy_(b["oc_all"].view(Hl, P, -1, D).transpose(0, 1))
            self.ex.heads_to_seq([st.b["oc_x"] for st in states], [st.b["oc"] for st in states])
        for st in states:
            b = st.b
            R = st.rows
            # attention output (+ the gated compressed branch) -> compact rows, quantized; out-projection with the
            # gated residual in the epilogue
            merge = {}
            if "o1" in b and meta.selection(n_all, i)["split"]:  # the dense-prefix pass, merged by log-sum-exp
                merge = {"o1": b["o1"], "lse1a": b["lse1a"], "lse1b": b["lse1b"], "lse2": b["lse2"]}
            if gate:
                ops.attn_gate_quant(b["ob"], b["g"], b["hs"], b["oc"], b["slot"], st.n_local, TILE, self._q(b["a"]),
                                    b["a_sf"], b["as"], R, **merge)
            else:
                ops.attn_gate_quant(b["ob"], None, None, None, b["slot"], st.n_local, TILE, self._q(b["a"]),
                                    b["a_sf"], b["as"], R, **merge)
            self._t(i, "gate", st, ob=b["ob"], a=b["a"], a_sf=b["a_sf"], sa=b["as"], g=b.get("g") if gate else None,
                    oc=b.get("oc") if gate else None, hs=b["hs"] if gate else None, h=b["h"] if gate else None,
                    h_sf=b["h_sf"] if gate else None)
            self._gemm(self._q(b["a"]), b["a_sf"], fz["o"], b["x"], row_scale=b["as"], residual=b["x"],
                       gate=tab[2])
            self._t(i, "out_proj", st, x=b["x"])
            # cross-attention: norm3 (affine LayerNorm as a table), q GEMM, per-tile E4M3 q, attention to the text
            ops.resid_norm_quant(b["x"], None, None, None, None, None, blk.norm3.shift, blk.norm3.scale, b["x"],
                                 self._q(b["h"]), b["h_sf"], b["hs"], blk.norm3.eps, norm="layer")
            self._t(i, "norm3", st, h=b["h"], h_sf=b["h_sf"], hs=b["hs"])
            self._gemm(self._q(b["h"]), b["h_sf"], fz["cq"], b["cq"])
            ops.head_tile_quant(b["cq"], b["hs"], b["tile_row0"], b["vbs"], blk.attn2.norm_q.weight, b["cqb"],
                                b["cqs"], None, H, st.n_local, blk.attn2.norm_q.eps)
            self._t(i, "cross_q", st, cq=b["cq"], cqb=b["cqb"], cqs=b["cqs"])
            ops.vsa_fp8_ex(b["cqb"], txt["kb"][i], txt["vb"][i], b["cob"], b["cidx"], b["cnum"], b["vbs"],
                           txt["vbs"], txt["vs"][i], txt["vs_head"][i], sm_scale * LOG2E, H, st.n_local, txt["n"],
                           st.rows_pad, txt["L"], qs=b["cqs"], ks=txt["ks"][i], idx_ld=txt["n"],
                           q_scale_ld=st.n_local, kv_scale_ld=txt["n"], shared_lists=True)
            ops.attn_gate_quant(b["cob"], None, None, None, b["slot"], st.n_local, TILE, self._q(b["a"]),
                                b["a_sf"], b["as"], R)
            self._t(i, "cross_attn", st, cob=b["cob"], a=b["a"], a_sf=b["a_sf"], sa=b["as"])
            self._gemm(self._q(b["a"]), b["a_sf"], fz["co"], b["x"], row_scale=b["as"], residual=b["x"],
                       gate=self.ones_c)
            self._t(i, "cross_out", st, x=b["x"])
            # FFN: norm2 + modulate + quant, fc_in with GELU-tanh, row quant, fc_out with the gated residual
            self._norm(st, blk.eps, tab[3:4], tab[4:5], i, "norm2")
            if self._ffn_state == "set":
                # fc_in + GELU-tanh with NVFP4 re-quantization in the epilogue under the block's fixed scale
                s_i = self.ffn_scales[i:i + 1]
                fi = fz["fc_in"]
                ops.gemm_nvfp4_requant(b["h"], b["h_sf"], fi["w"], fi["sf"], b["f"], b["f_sf"], s_i,
                                       scale_a=b["hs"], scale_b=fi["col"], act="gelu_tanh")
                self._t(i, "ffn_mid", st, f=b["f"], f_sf=b["f_sf"], fs=s_i)
                self._gemm(b["f"], b["f_sf"], fz["fc_out"], b["x"], alpha_dev=s_i, residual=b["x"], gate=tab[5])
            else:
                self._gemm(self._q(b["h"]), b["h_sf"], fz["fc_in"], b["u"], row_scale=b["hs"], act="gelu_tanh")
                if self.fp4:
                    ops.quant_nvfp4_rows(b["u"], b["f"], b["f_sf"], b["fs"])
                else:
                    ops.quant_fp8_rows(b["u"], b["f"].view(ops.FP8), b["fs"])
                if self._ffn_state == "recording":
                    ops.amax(b["u"], self._ffn_amax[i:i + 1])
                self._t(i, "ffn_mid", st, u=b["u"], f=b["f"], f_sf=b["f_sf"], fs=b["fs"])
                self._gemm(self._q(b["f"]), b["f_sf"], fz["fc_out"], b["x"], row_scale=b["fs"], residual=b["x"],
                           gate=tab[5])
            self._t(i, "fc_out", st, x=b["x"])
            # the next block's norm1 + modulate + quant
            if i + 1 < len(self.blocks):
                self._norm(st, self.blocks[i + 1].eps, tabs[i + 1, 0:1], tabs[i + 1, 1:2], i + 1)

    @staticmethod
    def _buf(b: dict, name: str, shape: tuple, dtype, fill=None) -> torch.Tensor:
        """A layout buffer created on first use (the dense-prefix buffers exist only for layouts that need them)."""
        t = b.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
            dev = b["x"].device
            t = b[name] = torch.empty(shape, device=dev, dtype=dtype) if fill is None else \
                torch.full(shape, fill, device=dev, dtype=dtype)
        return t

    def _dense_prefix(self, st: _RankState, n_pre_tiles: int, n_all: int, sm_scale: float) -> None:
        """The dense-prefix pass of one rank (the reference runs it on FlashAttention, __init__.py:304-324; here it
        is this library's attention kernel with every such key tile selected, over the same E4M3 operands): (a) the
        prefix query tiles against every key tile, in chunks of at most 1024 key tiles merged by log-sum-exp, and
        (b) every other query tile against the prefix key tiles. Writes ``o1`` [rows, H, 128] bf16 (compact rows) and
        the natural-log LSEs ``lse1a`` [H, prefix rows] / ``lse1b`` [H, other rows] that attn_gate_quant merges with
        the sparse pass (h3fast.cu:689-719)."""
        b = st.b
        H = self.heads
        L_MAX = 1024
        if n_pre_tiles > L_MAX:
            raise ValueError(f"{n_pre_tiles} prefix tiles: the attention kernel holds at most {L_MAX} per list")
        dev, i32 = self.dev, torch.int32
        rows_pad, R = st.rows_pad, st.rows
        n_pre_rows = int(st.lay.tile_row0[n_pre_tiles]) if n_pre_tiles < st.lay.n_ext else R
        n_q_a = n_pre_tiles + n_pre_tiles % 2
        coef = sm_scale * LOG2E
        args = dict(qs=b["qs_all"], ks=b["ks_all"], q_scale_ld=n_all, kv_scale_ld=n_all, qk_int8=self.qk_int8)
        # (a) prefix queries x every key tile, key chunks of <= L_MAX tiles
        outs = []
        for c0 in range(0, n_all, L_MAX):
            c1 = min(n_all, c0 + L_MAX)
            idx = torch.arange(c0, c1, device=dev, dtype=i32).repeat(H, n_q_a, 1).contiguous()
            num = torch.zeros(H, n_q_a, device=dev, dtype=i32)
            num[:, :n_pre_tiles] = c1 - c0
            out = torch.zeros(H, rows_pad, 128, device=dev, dtype=torch.bfloat16)
            lse = torch.full((H, rows_pad), -float("inf"), device=dev, dtype=torch.float32)
            ops.vsa_fp8_ex(b["qb_x"], b["kb_x"], b["vb_x"], out, idx, num, b["vbs_all"], b["vbs_all"], b["vs_all"],
                           b["vs_head"], coef, H, n_q_a, n_all, rows_pad, rows_pad, lse=lse, idx_ld=c1 - c0, **args)
            outs.append((out[:, :n_pre_tiles * TILE].float(), lse[:, :n_pre_tiles * TILE]))
        lses = torch.stack([lse for _, lse in outs])
        m = lses.amax(0)
        m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        w = torch.exp2(lses - m)
        den = w.sum(0)
        out_a = sum(wc[..., None] * o for wc, (o, _) in zip(w, outs)) / den.clamp_min(1e-30)[..., None]
        lse_a = torch.where(den > 0, m + torch.log2(den), torch.full_like(den, -float("inf")))
        # (b) every other query tile x the prefix key tiles
        idx = torch.arange(n_pre_tiles, device=dev, dtype=i32).repeat(H, n_all, 1).contiguous()
        num = torch.full((H, n_all), n_pre_tiles, device=dev, dtype=i32)
        num[:, :n_pre_tiles] = 0
        out_b = torch.zeros(H, rows_pad, 128, device=dev, dtype=torch.bfloat16)
        lse_b = torch.full((H, rows_pad), -float("inf"), device=dev, dtype=torch.float32)
        ops.vsa_fp8_ex(b["qb_x"], b["kb_x"], b["vb_x"], out_b, idx, num, b["vbs_all"], b["vbs_all"], b["vs_all"],
                       b["vs_head"], coef, H, n_all, n_all, rows_pad, rows_pad, lse=lse_b, idx_ld=n_pre_tiles, **args)
        out_b[:, :n_pre_tiles * TILE] = out_a.to(torch.bfloat16)
        lse_b[:, :n_pre_tiles * TILE] = lse_a
        slot = b["slot"].long()
        self._buf(b, "o1", (R, H, 128), torch.bfloat16).copy_(out_b[:, slot].transpose(0, 1))
        lse_rows = lse_b[:, slot] * math.log(2.0)  # log2 -> natural log
        self._buf(b, "lse1a", (H, n_pre_rows), torch.float32).copy_(lse_rows[:, :n_pre_rows])
        self._buf(b, "lse1b", (H, R - n_pre_rows), torch.float32).copy_(lse_rows[:, n_pre_rows:])

    # ------------------------------------------------------------------------------------------------- peer transport
    def _peer_streams(self) -> list:
        """One copy stream per destination rank (this one included), so the copies to different ranks can run on
        different copy engines."""
        if self._copy_streams is None:
            self._copy_streams = [torch.cuda.Stream(self.dev) for _ in range(self.ex.world)]
        return self._copy_streams

    def _peer_dims(self, st: _RankState) -> dict:
        return {"P": self.ex.world, "H": self.heads, "G": self.head_groups, "R": st.rows_pad, "D": self.head_dim}

    def _peer_send_heads(self, st: _RankState, stats: tuple) -> None:
        """Sequence -> heads over the peer transport, enqueued after the prologue: to every rank p (itself included),
        on p's copy stream, the tile statistics of p's heads into p's [Hl, n_all, ...] buffers at this rank's tile
        columns, then flag slot 0 (with ``stats_put``: all ranks' statistics and flags by one h3b_peer_put kernel on
        the compute stream instead); then head group by head group the Q/K/V planes of p's heads g*Hg .. into p's
        [planes, G, P, Hg, rows_pad, 128] buffer at (g, this rank), then flag slot 1 + g. Nothing here overwrites
        what a receiver still reads: a rank sends block i+1 only after its own gate quantizer of block i, which waited
        for every rank's attention outputs of block i, i.e. after every rank's last read of its receive buffers."""
        from ._lib import call
        ar, b, P, r = st.arena, st.b, self.ex.world, self.ex.sp.rank
        main = torch.cuda.current_stream(self.dev)
        ready = torch.cuda.Event()
        ready.record(main)
        e = self._epoch
        dims = self._peer_dims(st)
        parts = [("qkv_x", b["qkv_s"], b["qkv_s"].shape[0], 1)]
        if b["qkv_s"].shape[0] == 2:
            parts.append(("v_x", b["vb"], 1, b["vb"].element_size()))
        streams = self._peer_streams()
        put = self._peer_stats_put(st, stats) if self.stats_put else None
        if put is not None:
            # the tile statistics to every rank in one SM kernel on the compute stream, which raises each receiver's
            # flag slot 0 after the last byte; the Q/K/V planes (large) on the copy engines beside it
            arr, n, flags, n_flags, counter = put
            call("h3b_peer_put", arr, n, flags, n_flags, e, counter.data_ptr(), main.cuda_stream)
        for k in range(P):
            p = (r + 1 + k) % P
            cs = streams[p]
            cs.wait_event(ready)
            h = cs.cuda_stream
            if put is None:
                for nm in stats:
                    so, spitch, do, dpitch, w, rows = self._stats_plan(st, nm, p)
                    call("h3b_peer_copy2d", ar.ptr(p, nm + "_all", do), dpitch, b[nm].data_ptr() + so, spitch, w,
                         rows, h)
                call("h3b_peer_signal", ar.flag(p, 0, r), e, h)
            for g in range(self.head_groups):
                for region, src, planes, es in parts:
                    so, spitch, do, dpitch, w, rows = peer_copy_plan("qkv", r, p, g, dict(dims, planes=planes, es=es))
                    call("h3b_peer_copy2d", ar.ptr(p, region, do), dpitch, src.data_ptr() + so, spitch, w, rows, h)
                call("h3b_peer_signal", ar.flag(p, 1 + g, r), e, h)

    def _stats_plan(self, st: _RankState, nm: str, p: int) -> tuple:
        """peer_copy_plan of tile statistic ``nm`` from this rank to rank p."""
        T = st.b[nm][0, 0].numel()
        return peer_copy_plan("stats", self.ex.sp.rank, p, 0, dict(self._peer_dims(st), n=st.n_local, T=T, es=4))

    def _peer_stats_put(self, st: _RankState, stats: tuple):
        """h3b_peer_put's arguments for this rank's tile statistics to every rank (flag slot 0 of each), built once
        per layout; None when they exceed one put (more than 64 copies)."""
        from ._lib import PEER_PUT_MAX_COPIES, PeerCopy
        hit = st.b.get("_stats_put")
        if hit is not None and hit[0] == stats:
            return hit[1]
        P, r, ar, b = self.ex.world, self.ex.sp.rank, st.arena, st.b
        put = None
        if P * len(stats) <= PEER_PUT_MAX_COPIES:
            copies = []
            for p in range(P):
                for nm in stats:
                    so, spitch, do, dpitch, w, rows = self._stats_plan(st, nm, p)
                    copies.append(PeerCopy(ar.ptr(p, nm + "_all", do), b[nm].data_ptr() + so, dpitch, spitch, w, rows))
            flags = (ctypes.c_void_p * P)(*[ar.flag(p, 0, r) for p in range(P)])
            counter = torch.zeros(1, device=self.dev, dtype=torch.int32)
            put = ((PeerCopy * len(copies))(*copies), len(copies), flags, P, counter)
        b["_stats_put"] = (stats, put)
        return put

    def _peer_send_out(self, st: _RankState, g: int) -> None:
        """Heads -> sequence of head group g, enqueued after its attention: chunk p of the group's output (rank p's
        rows) into rank p's [H, rows_pad, 128] buffer at heads r*Hl + g*Hg .., then flag slot 1 + G + g."""
        from ._lib import call
        ar, b, P, r = st.arena, st.b, self.ex.world, self.ex.sp.rank
        main = torch.cuda.current_stream(self.dev)
        done = torch.cuda.Event()
        done.record(main)
        dims = dict(self._peer_dims(st), es=2)
        src = b["ob_x"].data_ptr()
        streams = self._peer_streams()
        for k in range(P):
            p = (r + 1 + k) % P
            cs = streams[p]
            cs.wait_event(done)
            h = cs.cuda_stream
            so, spitch, do, dpitch, w, rows = peer_copy_plan("out", r, p, g, dims)
            call("h3b_peer_copy2d", ar.ptr(p, "ob", do), dpitch, src + so, spitch, w, rows, h)
            call("h3b_peer_signal", ar.flag(p, 1 + self.head_groups + g, r), self._epoch, h)

    def _peer_wait(self, st: _RankState, slot: int, n_slots: int, name: str) -> None:
        """Bounded wait on the current stream until every rank's flags of slots [slot, slot + n_slots) hold this
        exchange's epoch (h3b_peer_wait: an expired wait sets the exchange status word, raised after the step)."""
        from ._lib import call
        main = torch.cuda.current_stream(self.dev)
        ar, r = st.arena, self.ex.sp.rank
        if self.ex.timing is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(main)
        call("h3b_peer_wait", ar.flag(r, slot, 0), n_slots * self.ex.world, self._epoch, 0, main.cuda_stream)
        if self.ex.timing is not None:
            e1.record(main)
            self.ex.timing.append((name, e0, e1))

    def _t(self, i: int, stage: str, st: _RankState, **tensors) -> None:
        if self.trace is not None:
            self.trace(i, stage, st.rank, tensors)

    def _q(self, t: torch.Tensor) -> torch.Tensor:
        return t if self.fp4 else t.view(ops.FP8)

    def _prologue(self, st: _RankState, blk) -> None:
        b = st.b
        C = self.hidden
        qkv = b["qkv"]
        ops.qkv_prologue8(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], b["hs"], b["tile_row0"], b["vbs"],
                          blk.attn.norm_q.weight, blk.attn.norm_k.weight, b["cos"], b["sin"], 1.0, 1.0, b["qb"],
                          b["kb"], b["vb"], b["vs"], None, b["qp"], b["kp"], b["vp"], self.heads, st.n_local, TILE,
                          blk.attn.norm_q.eps, qs_blk=b["qs"], ks_blk=b["ks"], qk_int8=self.qk_int8)


class Fp8BlockChain:
    """the FP8 DiT block MLP/projection chain without attention, on the same kernels as the block
    loop. LayerNorm (no affine) + modulate + per-token FP8 -> QKV 5120->15360 -> per-token FP8 of the V third ->
    out-projection 5120->5120 with the gated residual -> LayerNorm + modulate + FP8 -> fc_in 5120->13824 with GELU-tanh
    -> per-token FP8 -> fc_out 13824->5120 with the gated residual. Weights FP8 per output channel."""

    def __init__(self, qkv: list[QuantLinear], o: QuantLinear, fc_in: QuantLinear, fc_out: QuantLinear,
                 eps: float = 1e-6):
        self.qkv, self.o = _fused_rows(qkv), _fused_rows([o])
        self.fc_in, self.fc_out = _fused_rows([fc_in]), _fused_rows([fc_out])
        self.eps = eps
        self.C = o.out_features
        self.F = fc_in.out_features
        self.bufs: dict = {}
        self.trace = None

    @staticmethod
    def random(device="cuda", seed: int = 0, hidden: int = 5120, ffn: int = 13824) -> "Fp8BlockChain":
        g = torch.Generator(device=device)

        def randn(*shape, s):
            g.manual_seed(seed * 1_000_003 + s)
            return (torch.randn(*shape, device=device, generator=g) * 0.02).bfloat16()

        qkv = QuantLinear.pack_rows([randn(hidden, hidden, s=j) for j in range(3)], "fp8")
        (o,) = QuantLinear.pack_rows([randn(hidden, hidden, s=3)], "fp8")
        (f1,) = QuantLinear.pack_rows([randn(ffn, hidden, s=4)], "fp8")
        (f2,) = QuantLinear.pack_rows([randn(hidden, ffn, s=5)], "fp8")
        return Fp8BlockChain(qkv, o, f1, f2)

    def flop(self, rows: int) -> float:
        C, F = self.C, self.F
        return 2.0 * rows * (3 * C * C + C * C + 2 * C * F)

    def _buffers(self, rows: int, dev) -> dict:
        b = self.bufs.get(rows)
        if b is None:
            C, F = self.C, self.F
            b = self.bufs[rows] = {
                "h": torch.empty(rows, C, device=dev, dtype=ops.FP8), "hs": torch.empty(rows, device=dev),
                "qkv": torch.empty(rows, 3 * C, device=dev, dtype=torch.bfloat16),
                "a": torch.empty(rows, C, device=dev, dtype=ops.FP8), "as": torch.empty(rows, device=dev),
                "u": torch.empty(rows, F, device=dev, dtype=torch.bfloat16),
                "f": torch.empty(rows, F, device=dev, dtype=ops.FP8), "fs": torch.empty(rows, device=dev)}
        return b

    def _t(self, stage, **tensors):
        if self.trace is not None:
            self.trace(stage, tensors)

    def __call__(self, x: torch.Tensor, tabs: torch.Tensor, check: bool = True) -> torch.Tensor:
        """x bf16 [rows, 5120] updated in place; tabs bf16 [6, 5120] = shift, scale, gate (attention half), shift,
        scale, gate (MLP half). ``check``: read the GEMMs' device status word after the last GEMM (one host sync) and
        raise on a failure."""
        rows, C = x.shape
        b = self._buffers(rows, x.device)
        ops.resid_norm_quant(x, None, None, None, None, None, tabs[0:1], tabs[1:2], x, b["h"], None, b["hs"],
                             self.eps, norm="layer")
        self._t("norm1", x=x, h=b["h"], hs=b["hs"])
        ops.gemm_fp8(b["h"], self.qkv["w"], b["qkv"], scale_a=b["hs"], scale_b=self.qkv["col"])
        ops.quant_fp8_rows(b["qkv"][:, 2 * C:], b["a"], b["as"])
        self._t("qkv", qkv=b["qkv"], a=b["a"], sa=b["as"])
        ops.gemm_fp8(b["a"], self.o["w"], x, scale_a=b["as"], scale_b=self.o["col"], residual=x, gate=tabs[2])
        self._t("out_proj", x=x)
        ops.resid_norm_quant(x, None, None, None, None, None, tabs[3:4], tabs[4:5], x, b["h"], None, b["hs"],
                             self.eps, norm="layer")
        self._t("norm2", h=b["h"], hs=b["hs"])
        ops.gemm_fp8(b["h"], self.fc_in["w"], b["u"], scale_a=b["hs"], scale_b=self.fc_in["col"], act="gelu_tanh")
        ops.quant_fp8_rows(b["u"], b["f"], b["fs"])
        self._t("ffn_mid", u=b["u"], f=b["f"], fs=b["fs"])
        ops.gemm_fp8(b["f"], self.fc_out["w"], x, scale_a=b["fs"], scale_b=self.fc_out["col"], residual=x,
                     gate=tabs[5])
        self._t("fc_out", x=x)
        if check and not torch.cuda.is_current_stream_capturing():
            ops.check_status(x.device)
        return x


class GraphedForward:
    """``H3FastRunner.forward`` captured once into a CUDA graph and replayed (one rank): every launch of the 50-block
    step -- kernels, the side-stream branch, the torch glue -- is one graph launch, with no per-launch host work.

    The graph reads its inputs from static buffers: ``__call__(packed, temb)`` copies the new latent and timestep
    embedding in and replays. The text context, the metadata, rotary tables and the reduction plan are fixed at
    capture (the text keys/values are projected before the capture and cached; a new context needs a new
    ``GraphedForward``). Returns the static output tensor, overwritten by the next replay."""

    def __init__(self, runner: H3FastRunner, packed: torch.Tensor, temb: torch.Tensor, meta: VsaMeta,
                 context: torch.Tensor, rotary=None, reduction: TokenReduction | None = None):
        if runner.ex.world != 1:
            raise ValueError("GraphedForward captures one rank")
        self.runner = runner
        self.packed = packed.clone()
        self.temb = temb.clone()
        self.context = context
        args = (None, rotary, meta)
        kw = {"context": context, "reduction": reduction}
        runner.forward(self.packed, self.temb, *args, **kw)  # layouts, text cache, kernel attributes: outside capture
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = runner.forward(self.packed, self.temb, *args, **kw)
        torch.cuda.synchronize()

    def __call__(self, packed: torch.Tensor, temb: torch.Tensor | None = None) -> torch.Tensor:
        self.packed.copy_(packed)
        if temb is not None:
            self.temb.copy_(temb)
        self.graph.replay()
        if self.runner.check_status:
            ops.check_status(self.runner.dev)
        return self.out
