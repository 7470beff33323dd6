"""Weight-load path: dense checkpoints (safetensors) to packed FP8 / NVFP4 linears, FastVideo's in-place FP8 conversion
of a module tree, and LoRA adapters merged on the base weight's FP8 grid.

- ``load_dit_checkpoint`` / ``save_dit_checkpoint``: the on-disk boundary of ``DiTModel`` (names and shapes of
  ``DiTModel.checkpoint_specs``). Tensors are read one at a time (``safetensors.safe_open``), staged through two
  page-locked host buffers and copied on their own stream, and packed on the device block by block by the h3b packing
  kernels, so neither the whole dense model nor a second host copy of it is ever resident.
- ``convert_model_to_fp8``: ``convert_model_to_fp8`` of patches/fastvideo-a01c50a.patch:397-471 for a torch module
  tree -- every FP8-tagged linear gets ``_fp8_weight`` / ``_fp8_weight_scale`` (``quantize_fp8_weight``, :384-394) and
  loses its dense ``weight``; with ``keep_sources`` the dense weights are kept in one page-locked host slab per dtype
  (``_fp8_source``) for LoRA merging (:405-416).
- ``LoraMerger``: ``H3FastRunner._merged_fp8`` (fastvideo/models/dits/h3fast/__init__.py:354-376) -- the adapter's
  ``scale * B @ A`` added to the dense source in float32 (a plain cuBLAS GEMM), then ``_on_grid`` (:82-92) on the base
  weight's scales by ``ops.quant_fp8_on_grid``; cached per layer until the adapter or its strength changes.

There is no CPU path: the packing and grid kernels are the h3b library's (``ops``), which raises without it.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Callable, Mapping

import torch

from . import ops
from .model import DiTConfig, DiTModel, QuantLinear

# --------------------------------------------------------------------------------------------- checkpoints


def save_dit_checkpoint(tensors: Mapping[str, torch.Tensor], path: str | Path,
                        config: DiTConfig | None = None) -> None:
    """Writes dense tensors (names of ``DiTModel.checkpoint_specs(config)``, any device) as one safetensors file."""
    from safetensors.torch import save_file

    specs = DiTModel.checkpoint_specs(config) if config is not None else None
    if specs is not None:
        missing = sorted(set(specs) - set(tensors))
        if missing:
            raise ValueError(f"checkpoint lacks {len(missing)} tensors, e.g. {missing[:3]}")
    save_file({k: v.detach().to("cpu").contiguous() for k, v in tensors.items()}, str(path))


class _PinnedStage:
    """Two page-locked staging buffers (each grown to the largest tensor) and a copy stream for host -> device copies
    of checkpoint tensors: the file read and host copy of tensor i+1 overlap the device copy of tensor i, and the
    packing kernels on the current stream wait for their tensor's copy on the device, not on the host."""

    def __init__(self, device: torch.device) -> None:
        self.bufs: list[torch.Tensor | None] = [None, None]
        self.events: list[torch.cuda.Event | None] = [None, None]
        self.i = 0
        self.stream = torch.cuda.Stream(device)

    def to_device(self, t: torch.Tensor, device: torch.device) -> torch.Tensor:
        slot = self.i % 2
        self.i += 1
        if self.events[slot] is not None:
            self.events[slot].synchronize()  # the device copy that last read this buffer has finished
        nbytes = t.numel() * t.element_size()
        if self.bufs[slot] is None or self.bufs[slot].numel() < nbytes:
            self.bufs[slot] = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        staged = self.bufs[slot][:nbytes].view(t.dtype).view(t.shape)
        staged.copy_(t)
        cur = torch.cuda.current_stream(device)
        with torch.cuda.stream(self.stream):
            # allocated on the copy stream (its memory is reused in that stream's order), recorded on the current
            # stream (not reused before the packing kernels there have read it)
            out = torch.empty(t.shape, dtype=t.dtype, device=device)
            out.copy_(staged, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self.events[slot] = ev
        cur.wait_event(ev)
        out.record_stream(cur)
        return out


def load_dit_checkpoint(path: str | Path, config: DiTConfig | None = None,
                        device: str | torch.device = "cuda") -> DiTModel:
    """A packed ``DiTModel`` (``config.fmt``: NVFP4 or FP8 per channel) from a dense safetensors checkpoint.

    Every tensor of ``DiTModel.checkpoint_specs(config)`` must be present with its shape (float32, float16 or bf16;
    cast to bf16 on the device before packing, as FastVideo loads a bf16 DiT before converting it)."""
    from safetensors import safe_open

    cfg = config or DiTConfig()
    dev = torch.device(device)
    stage = _PinnedStage(dev)
    with safe_open(str(path), framework="pt", device="cpu") as f:
        have = set(f.keys())
        missing = sorted(set(DiTModel.checkpoint_specs(cfg)) - have)
        if missing:
            raise ValueError(f"{path}: {len(missing)} tensors missing, e.g. {missing[:3]}")

        def get(name: str) -> torch.Tensor:
            return stage.to_device(f.get_tensor(name), dev)

        model = DiTModel.from_dense(cfg, get, dev)
    torch.cuda.current_stream(dev).synchronize()  # the staging buffers are released after every copy has landed
    return model


# --------------------------------------------------------------------------------------------- FP8 module conversion


def _is_fastvideo_fp8(qm: Any) -> bool:
    return type(qm).__name__ == "FP8QuantizeMethod"


def _page_locked(numel_by_dtype: dict[torch.dtype, int]) -> dict[torch.dtype, torch.Tensor]:
    """One host slab per dtype, page-locked with cudaHostRegister (the pinned caching allocator would round each slab
    up to a power of two; patch:384-396 takes the same route)."""
    slabs = {}
    for dtype, numel in numel_by_dtype.items():
        slab = torch.empty(numel, dtype=dtype)
        if torch.cuda.is_available():
            err = torch.cuda.cudart().cudaHostRegister(slab.data_ptr(), slab.numel() * slab.element_size(), 0)
            if int(err) != 0:
                raise RuntimeError(f"cudaHostRegister failed ({int(err)}) for a {slab.numel()}-element slab")
        slabs[dtype] = slab
    return slabs


@torch.no_grad()
def convert_model_to_fp8(model: torch.nn.Module, *, keep_sources: bool = False,
                         is_fp8: Callable[[Any], bool] = _is_fastvideo_fp8,
                         quantize: Callable[..., tuple[torch.Tensor, torch.Tensor]] | None = None) -> int:
    """Quantizes every FP8-tagged linear of ``model`` in place (patch:397-471): registers ``_fp8_weight`` (e4m3
    [out, in]) and ``_fp8_weight_scale`` (float32, per output channel or per tensor per the quant method's
    ``granularity``) and drops the dense ``weight``. ``keep_sources`` keeps each dense weight as ``_fp8_source`` in a
    page-locked host slab (one per dtype) for ``LoraMerger``. ``quantize(weight, granularity)`` defaults to the h3b
    packing kernel (``ops.quantize_fp8_weight``). Returns the number of converted modules."""
    quantize = quantize or ops.quantize_fp8_weight
    modules = [m for m in model.modules()
               if is_fp8(getattr(m, "quant_method", None)) and getattr(m, "weight", None) is not None]
    sources = None
    if keep_sources:
        sizes: dict[torch.dtype, int] = {}
        for m in modules:
            sizes[m.weight.dtype] = sizes.get(m.weight.dtype, 0) + m.weight.numel()
        sources = {dt: [slab, 0] for dt, slab in _page_locked(sizes).items()}
    for m in modules:
        w = m.weight
        if sources is not None:
            slab = sources[w.dtype]
            m._fp8_source = slab[0][slab[1]:slab[1] + w.numel()].view(w.shape).copy_(w.detach())
            slab[1] += w.numel()
        wq, ws = quantize(w.detach().contiguous(), getattr(m.quant_method, "granularity", "tensor"))
        m.register_buffer("_fp8_weight", wq, persistent=False)
        m.register_buffer("_fp8_weight_scale", ws, persistent=False)
        m._parameters.pop("weight", None)
    return len(modules)


# --------------------------------------------------------------------------------------------- LoRA on the FP8 grid


def lora_scale(strength: float, alpha: float, rank: int) -> float:
    """The adapter factor of ``_adapter`` (__init__.py:63-73): strength * alpha / rank (strength when alpha == rank)."""
    return strength * (float(alpha) / float(rank) if alpha != rank else 1.0)


class LoraMerger:
    """FP8 weights with a LoRA adapter merged in, cached per layer (``_merged_fp8``, __init__.py:354-376).

    ``merged_fp8(layer, source, A, B, scale, base_scale, key)`` returns ``(e4m3 [N, K], float32 scale)`` of
    ``source + scale * B @ A`` on the grid ``base_scale``; the cache entry of ``layer`` is rebuilt when ``key`` (the
    reference keys by adapter path and strength) differs from the cached one."""

    def __init__(self, device: str | torch.device = "cuda") -> None:
        self.device = torch.device(device)
        self._merged: dict[int, tuple] = {}

    @torch.no_grad()
    def merged_fp8(self, layer: Any, source: torch.Tensor, A: torch.Tensor, B: torch.Tensor, scale: float,
                   base_scale: torch.Tensor, key: Any) -> tuple[torch.Tensor, torch.Tensor]:
        entry = self._merged.get(id(layer))
        if entry is None or not _same_key(entry[0], key):
            merged = source.to(self.device, non_blocking=True).float()
            merged.addmm_(B.to(self.device, torch.float32), A.to(self.device, torch.float32), alpha=scale)
            wq, ws = ops.quant_fp8_on_grid(merged, base_scale.to(self.device))
            del merged
            entry = self._merged[id(layer)] = (key, wq, ws)
        return entry[1], entry[2]

    def clear(self) -> None:
        self._merged.clear()


def _same_key(a: Any, b: Any) -> bool:
    if isinstance(a, tuple) and isinstance(b, tuple):
        return len(a) == len(b) and all(x is y or (not torch.is_tensor(x) and x == y) for x, y in zip(a, b))
    return a is b or (not torch.is_tensor(a) and a == b)


def merge_lora_into(lin: QuantLinear, merger: LoraMerger, source: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
                    strength: float, alpha: float, rank: int, key: Any = None) -> None:
    """Points an FP8 ``QuantLinear`` at its weight with the adapter merged (the base weight and scale are kept as
    ``_fp8_base`` and restored by ``unmerge_lora``). A runner built before the merge picks the new weights up after
    ``H3FastRunner.refresh_weights()``."""
    if lin.fmt != "fp8":
        raise ValueError("LoRA merging is defined on the FP8 grid (NVFP4 linears take adapters as a side branch)")
    if not hasattr(lin, "_fp8_base"):
        lin._fp8_base = (lin._fp8_weight, lin._fp8_weight_scale)
    s = lora_scale(strength, alpha, rank)
    wq, ws = merger.merged_fp8(lin, source, A, B, s, lin._fp8_base[1], key if key is not None else (id(A), id(B), s))
    lin._fp8_weight, lin._fp8_weight_scale = wq, ws


def unmerge_lora(lin: QuantLinear) -> None:
    if hasattr(lin, "_fp8_base"):
        lin._fp8_weight, lin._fp8_weight_scale = lin._fp8_base
        del lin._fp8_base
