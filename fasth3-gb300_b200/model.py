"""The DiT the block runner executes: the quantized Linear surface and the block attributes the reference runner reads
(fastvideo/models/dits/h3fast/__init__.py:119-126, 164-171, 378-404), for BASELINE's architecture -- hidden 5120,
40 heads x 128, FFN 13824 with GELU-tanh, adaLN-zero modulation from the timestep, self-attention with per-head
QK-RMSNorm and 3D RoPE, cross-attention to 512 text tokens of width 4096.

Weights come from a dense checkpoint (``weights.load_dit_checkpoint``, names of ``DiTModel.checkpoint_specs``) or are
random-init N(0, 0.02) (``DiTModel.random``: generated on the device from per-tensor seeds, so that every rank of a
sequence-parallel job holds the same model); either way they are packed once at construction, block by block, the way
FastVideo's quant methods pack a checkpoint: NVFP4 (``_nvfp4_weight`` [N, K/2], ``_nvfp4_weight_scale`` 128x4 [pad128(N), K/16], ``_nvfp4_alpha``) or FP8
per output channel (``_fp8_weight`` [N, K], ``_fp8_weight_scale`` [N]; patches/fastvideo-a01c50a.patch:384-394, 459-460).
The q/k/v (and cross-attention k/v) linears of a block are packed into one buffer and exposed as row views of it, so
the runner issues one GEMM for them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import ops


@dataclass
class DiTConfig:
    hidden: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    text_dim: int = 4096
    text_len: int = 512
    blocks: int = 50
    freq_dim: int = 256
    eps: float = 1e-6
    fmt: str = "nvfp4"  # "nvfp4" | "fp8"
    # self-attention gate-compress branch (VSA's compressed branch gated per channel, FastVideo's to_gate_compress);
    # BASELINE's DiT has none
    gate_compress: bool = False


class QuantLinear:
    """A packed linear layer with the attribute names H3FastRunner._gemm reads."""

    def __init__(self, out_features: int, in_features: int, fmt: str):
        self.out_features, self.in_features, self.fmt = out_features, in_features, fmt
        self.bias = None

    @staticmethod
    def pack_rows(dense: list[torch.Tensor], fmt: str) -> list["QuantLinear"]:
        """Packs several dense bf16 weights with the same K into one buffer; returns one QuantLinear per weight, each a
        row view of the shared packing (NVFP4: one global scale per weight, kept per view as ``_nvfp4_alpha``)."""
        K = dense[0].shape[1]
        Ns = [w.shape[0] for w in dense]
        if any(n % 128 for n in Ns):
            raise ValueError("pack_rows: every weight needs a multiple of 128 rows (block-scale atoms)")
        dev = dense[0].device
        out = []
        if fmt == "nvfp4":
            wq = torch.empty(sum(Ns), K // 2, device=dev, dtype=torch.uint8)
            wsf = torch.empty(sum(Ns), K // 16, device=dev, dtype=torch.uint8)
            r = 0
            for w, n in zip(dense, Ns):
                q, sf, s = ops.pack_nvfp4_weight(w)
                wq[r:r + n].copy_(q)
                wsf[r:r + n].copy_(sf)
                lin = QuantLinear(n, K, fmt)
                lin._nvfp4_weight, lin._nvfp4_weight_scale, lin._nvfp4_alpha = wq[r:r + n], wsf[r:r + n], s
                out.append(lin)
                r += n
        elif fmt == "fp8":
            wq = torch.empty(sum(Ns), K, device=dev, dtype=ops.FP8)
            ws = torch.empty(sum(Ns), device=dev, dtype=torch.float32)
            r = 0
            for w, n in zip(dense, Ns):
                q, s = ops.quantize_fp8_weight(w, "channel")
                wq[r:r + n].copy_(q)
                ws[r:r + n].copy_(s)
                lin = QuantLinear(n, K, fmt)
                lin._fp8_weight, lin._fp8_weight_scale = wq[r:r + n], ws[r:r + n]
                out.append(lin)
                r += n
        else:
            raise ValueError(f"unknown weight format {fmt!r}")
        return out


@dataclass
class RMSNorm:
    weight: torch.Tensor
    eps: float


@dataclass
class LayerNormAffine:
    """LayerNorm with weight and bias, applied as adaLN tables: shift = bias, scale = weight - 1."""
    shift: torch.Tensor  # bf16 [1, C]
    scale: torch.Tensor  # bf16 [1, C]
    eps: float


class Attention:
    def __init__(self, to_q, to_k, to_v, to_out, norm_q, norm_k, heads, head_dim):
        self.to_q, self.to_k, self.to_v, self.to_out = to_q, to_k, to_v, to_out
        self.norm_q, self.norm_k = norm_q, norm_k
        self.num_attention_heads, self.attention_head_dim = heads, head_dim
        self.to_gate_compress = None


class FeedForward:
    def __init__(self, fc_in, fc_out):
        self.fc_in, self.fc_out = fc_in, fc_out


@dataclass
class DiTBlock:
    attn: Attention
    attn2: Attention             # cross-attention to the text tokens
    norm3: LayerNormAffine       # before the cross-attention
    ff: FeedForward
    scale_shift_table: torch.Tensor  # bf16 [6, C]: per-block adaLN offsets added to the timestep projection
    eps: float


@dataclass
class DiTModel:
    config: DiTConfig
    transformer_blocks: list[DiTBlock]
    time_mlp: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]  # W1 [C, F], b1, W2 [C, C], b2 (bf16)
    time_proj: tuple[torch.Tensor, torch.Tensor]  # W [6C, C], b [6C]
    extra: dict = field(default_factory=dict)

    def timestep_embedding(self, t: float) -> torch.Tensor:
        """Sinusoidal embedding of t*1000 (freq_dim) -> MLP (SiLU) -> temb bf16 [1, C]."""
        cfg = self.config
        dev = self.time_proj[0].device
        half = cfg.freq_dim // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=dev, dtype=torch.float32) / half)
        arg = (t * 1000.0) * freqs
        emb = torch.cat([torch.cos(arg), torch.sin(arg)])[None].to(torch.bfloat16)
        w1, b1, w2, b2 = self.time_mlp
        h = torch.nn.functional.silu(emb @ w1.t() + b1)
        return h @ w2.t() + b2

    def adaln_tables(self, temb: torch.Tensor) -> torch.Tensor:
        """bf16 [blocks, 6, C]: (shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp) per block, the
        timestep projection of SiLU(temb) plus each block's own table (adaLN-zero)."""
        w, b = self.time_proj
        e0 = (torch.nn.functional.silu(temb) @ w.t() + b).view(6, -1)
        return torch.stack([blk.scale_shift_table + e0 for blk in self.transformer_blocks])

    @staticmethod
    def checkpoint_specs(config: DiTConfig | None = None) -> dict[str, tuple[int, ...]]:
        """Names and shapes of the dense tensors a checkpoint of this DiT holds (FastVideo-style names: blocks under
        ``transformer_blocks.{i}``, the self-attention as ``attn``, the cross-attention as ``attn2``)."""
        cfg = config or DiTConfig()
        C, F, T, D = cfg.hidden, cfg.ffn, cfg.text_dim, cfg.head_dim
        specs: dict[str, tuple[int, ...]] = {
            "time_embedder.linear_1.weight": (C, cfg.freq_dim), "time_embedder.linear_1.bias": (C,),
            "time_embedder.linear_2.weight": (C, C), "time_embedder.linear_2.bias": (C,),
            "time_proj.weight": (6 * C, C), "time_proj.bias": (6 * C,)}
        for i in range(cfg.blocks):
            p = f"transformer_blocks.{i}."
            for a, kv in (("attn", C), ("attn2", T)):
                specs.update({p + f"{a}.to_q.weight": (C, C), p + f"{a}.to_k.weight": (C, kv),
                              p + f"{a}.to_v.weight": (C, kv), p + f"{a}.to_out.weight": (C, C),
                              p + f"{a}.norm_q.weight": (D,), p + f"{a}.norm_k.weight": (D,)})
            specs.update({p + "norm3.weight": (C,), p + "norm3.bias": (C,), p + "ff.fc_in.weight": (F, C),
                          p + "ff.fc_out.weight": (C, F), p + "scale_shift_table": (6, C)})
            if cfg.gate_compress:
                specs[p + "attn.to_gate_compress.weight"] = (C, C)
        return specs

    @staticmethod
    def from_dense(config: DiTConfig, get, device: str | torch.device = "cuda") -> "DiTModel":
        """Builds the model from dense tensors: ``get(name)`` returns the tensor named in ``checkpoint_specs`` (any
        device, any float dtype; it is cast to bf16 and moved to ``device``). Linears are packed block by block as
        they arrive (``config.fmt``), so at most one block's dense weights are on the device at a time."""
        cfg = config
        specs = DiTModel.checkpoint_specs(cfg)

        def t(name: str) -> torch.Tensor:
            x = get(name)
            if tuple(x.shape) != specs[name]:
                raise ValueError(f"{name}: shape {tuple(x.shape)}, expected {specs[name]}")
            return x.to(device=device, dtype=torch.bfloat16).contiguous()

        blocks = []
        for i in range(cfg.blocks):
            p = f"transformer_blocks.{i}."
            q, k, v = QuantLinear.pack_rows([t(p + f"attn.to_{n}.weight") for n in "qkv"], cfg.fmt)
            (o,) = QuantLinear.pack_rows([t(p + "attn.to_out.weight")], cfg.fmt)
            (cq,) = QuantLinear.pack_rows([t(p + "attn2.to_q.weight")], cfg.fmt)
            ck, cv = QuantLinear.pack_rows([t(p + "attn2.to_k.weight"), t(p + "attn2.to_v.weight")], cfg.fmt)
            (co,) = QuantLinear.pack_rows([t(p + "attn2.to_out.weight")], cfg.fmt)
            (f1,) = QuantLinear.pack_rows([t(p + "ff.fc_in.weight")], cfg.fmt)
            (f2,) = QuantLinear.pack_rows([t(p + "ff.fc_out.weight")], cfg.fmt)
            attn = Attention(q, k, v, o, RMSNorm(t(p + "attn.norm_q.weight"), cfg.eps),
                             RMSNorm(t(p + "attn.norm_k.weight"), cfg.eps), cfg.heads, cfg.head_dim)
            if cfg.gate_compress:
                (attn.to_gate_compress,) = QuantLinear.pack_rows([t(p + "attn.to_gate_compress.weight")], cfg.fmt)
            attn2 = Attention(cq, ck, cv, co, RMSNorm(t(p + "attn2.norm_q.weight"), cfg.eps),
                              RMSNorm(t(p + "attn2.norm_k.weight"), cfg.eps), cfg.heads, cfg.head_dim)
            # affine LayerNorm as an adaLN table: shift = bias, scale = weight - 1 (exact in float32, rounded to bf16)
            w3 = t(p + "norm3.weight").float()
            norm3 = LayerNormAffine(t(p + "norm3.bias").reshape(1, -1), (w3 - 1.0).to(torch.bfloat16).reshape(1, -1),
                                    cfg.eps)
            blocks.append(DiTBlock(attn, attn2, norm3, FeedForward(f1, f2), t(p + "scale_shift_table"), cfg.eps))
        time_mlp = (t("time_embedder.linear_1.weight"), t("time_embedder.linear_1.bias"),
                    t("time_embedder.linear_2.weight"), t("time_embedder.linear_2.bias"))
        time_proj = (t("time_proj.weight"), t("time_proj.bias"))
        return DiTModel(cfg, blocks, time_mlp, time_proj)

    @staticmethod
    def random_dense(config: DiTConfig | None = None, device: str | torch.device = "cuda", seed: int = 0):
        """``get(name)`` for ``from_dense``: every tensor N(0, 0.02) (norm weights 1 + N(0, 0.1), adaLN tables and
        norm3's offsets N(0, 0.1), time biases 0) from its own seed on ``device``, so any subset can be drawn in any
        order and every rank of a sequence-parallel job draws the same model."""
        cfg = config or DiTConfig()
        specs = DiTModel.checkpoint_specs(cfg)
        names = list(specs)
        g = torch.Generator(device=device)

        def get(name: str) -> torch.Tensor:
            g.manual_seed(seed * 1_000_003 + names.index(name))
            leaf = name.rsplit(".", 1)[-1]
            if name.startswith("time") and leaf == "bias":
                return torch.zeros(specs[name], device=device, dtype=torch.bfloat16)
            std = 0.1 if ("norm" in name or leaf == "scale_shift_table" or leaf == "bias") else 0.02
            x = torch.randn(*specs[name], device=device, generator=g, dtype=torch.float32) * std
            if "norm" in name and leaf == "weight":
                x = 1.0 + x
            return x.to(torch.bfloat16)

        return get

    @staticmethod
    def random(config: DiTConfig | None = None, device: str | torch.device = "cuda", seed: int = 0) -> "DiTModel":
        """Random-init weights (no checkpoints): ``from_dense`` over ``random_dense``."""
        cfg = config or DiTConfig()
        return DiTModel.from_dense(cfg, DiTModel.random_dense(cfg, device, seed), device)
