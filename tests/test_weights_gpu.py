"""Weight-load path on the GPU: the FP8 grid kernel against the reference's ``_on_grid`` (golden vectors), a dense
safetensors checkpoint loading to the same packed bytes as the in-memory model, and a LoRA adapter merged into an FP8
linear (grid codes bit-exact against the oracle on the same merged weight, GEMM within FP8 tolerance of the fp32
merged weight, the runner picking it up and returning bit-exactly to the base model when it is removed)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import lora as ol

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "lora_on_grid.npz"


@pytest.fixture(scope="module")
def pk(h3b):
    return h3b.model, h3b.runner, h3b.weights


@pytest.mark.parametrize("case", ["lora_rows", "lora_tensor_own", "lora_tensor_grid"])
def test_on_grid_kernel_matches_reference(ops, case):
    d = np.load(GOLDEN)
    merged = torch.from_numpy(d[f"{case}.merged"]).to(DEV)
    base = torch.from_numpy(d[f"{case}.base_scale"]).to(DEV)
    wq, ws = ops.quant_fp8_on_grid(merged, base)
    assert np.array_equal(wq.view(torch.uint8).cpu().numpy(), d[f"{case}.q"])
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), d[f"{case}.s"].view(np.uint32))


def test_on_grid_kernel_large_rows(ops):
    """A full-size merged weight (5120 x 13824, one row in 11 outgrowing its grid) against the oracle."""
    g = torch.Generator(device=DEV).manual_seed(7)
    w = torch.randn(5120, 13824, device=DEV, generator=g) * 0.02
    base = (w.abs().amax(dim=1) / 448.0).clamp(min=1e-12)
    w[::11] *= 1.2
    wq, ws = ops.quant_fp8_on_grid(w, base)
    q, s = ol.on_grid(w.cpu().numpy(), base.cpu().numpy())
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), s.view(np.uint32))
    assert np.array_equal(wq.view(torch.uint8).cpu().numpy(), q)


@pytest.mark.parametrize("fmt", ["nvfp4", "fp8"])
def test_checkpoint_loads_to_the_same_packing(tmp_path, pk, fmt):
    model, _, weights = pk
    cfg = model.DiTConfig(blocks=2, hidden=256, heads=2, ffn=512, text_dim=256, fmt=fmt)
    get = model.DiTModel.random_dense(cfg, DEV, seed=5)
    dense = {n: get(n) for n in model.DiTModel.checkpoint_specs(cfg)}
    path = tmp_path / "dit.safetensors"
    weights.save_dit_checkpoint(dense, path, cfg)
    got = weights.load_dit_checkpoint(path, cfg, DEV)
    want = model.DiTModel.random(cfg, DEV, seed=5)
    names = ("_nvfp4_weight", "_nvfp4_weight_scale", "_nvfp4_alpha") if fmt == "nvfp4" else (
        "_fp8_weight", "_fp8_weight_scale")
    for bg, bw in zip(got.transformer_blocks, want.transformer_blocks):
        for lg, lw in [(bg.attn.to_q, bw.attn.to_q), (bg.attn.to_v, bw.attn.to_v), (bg.attn2.to_k, bw.attn2.to_k),
                       (bg.ff.fc_in, bw.ff.fc_in), (bg.ff.fc_out, bw.ff.fc_out)]:
            for a in names:
                assert torch.equal(getattr(lg, a).view(torch.uint8), getattr(lw, a).view(torch.uint8)), a
        assert torch.equal(bg.norm3.scale, bw.norm3.scale) and torch.equal(bg.scale_shift_table, bw.scale_shift_table)
        assert torch.equal(bg.attn.norm_k.weight, bw.attn.norm_k.weight)
    assert torch.equal(got.time_proj[0], want.time_proj[0])


def test_lora_merge_fp8_linear_and_runner(pk, ops):
    model, runner, weights = pk
    cfg = model.DiTConfig(blocks=1, fmt="fp8")
    m = model.DiTModel.random(cfg, DEV, seed=2)
    grid = (8, 16, 16)
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(1, grid[0] * grid[1] * grid[2], cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    r = runner.H3FastRunner(m)
    base_out = r.forward(x, temb, None, None, meta, context=ctx).clone()

    lin = m.transformer_blocks[0].attn.to_out
    base_w, base_s = lin._fp8_weight, lin._fp8_weight_scale
    src = model.DiTModel.random_dense(cfg, DEV, seed=2)("transformer_blocks.0.attn.to_out.weight")
    rank = 16
    A = (torch.randn(rank, cfg.hidden, device=DEV, generator=g) * 0.05).bfloat16()
    B = (torch.randn(cfg.hidden, rank, device=DEV, generator=g) * 0.02).bfloat16()
    B[::9] *= 30.0  # some rows outgrow the grid
    merger = weights.LoraMerger(DEV)
    weights.merge_lora_into(lin, merger, src.cpu().pin_memory(), A, B, strength=0.9, alpha=32, rank=rank)
    s = weights.lora_scale(0.9, 32, rank)

    # the grid step, bit-exact on the same fp32 merged weight
    merged = src.float()
    merged.addmm_(B.float(), A.float(), alpha=s)
    q, qs = ol.on_grid(merged.cpu().numpy(), base_s.cpu().numpy())
    assert np.array_equal(lin._fp8_weight.view(torch.uint8).cpu().numpy(), q)
    assert np.array_equal(lin._fp8_weight_scale.cpu().numpy().view(np.uint32), qs.view(np.uint32))
    assert 0 < int((lin._fp8_weight_scale != base_s).sum()) < cfg.hidden

    # the merged FP8 weight stays within E4M3 rounding of the fp32 merged weight, and a GEMM with it matches
    # dequantize-then-matmul in fp32 (rel-Frobenius 1e-3, the FP8 linear's bar)
    deq_w = lin._fp8_weight.float() * lin._fp8_weight_scale[:, None]
    assert float((deq_w - merged).norm() / merged.norm()) < 5e-2
    a = torch.randn(512, cfg.hidden, device=DEV, generator=g).bfloat16()
    aq = torch.empty(512, cfg.hidden, device=DEV, dtype=ops.FP8)
    sa = torch.empty(512, device=DEV)
    ops.quant_fp8_rows(a, aq, sa)
    y = torch.empty(512, cfg.hidden, device=DEV, dtype=torch.bfloat16)
    ops.gemm_fp8(aq, lin._fp8_weight, y, scale_a=sa, scale_b=lin._fp8_weight_scale)
    ref = ((aq.double() * sa.double()[:, None]) @ deq_w.double().t()).bfloat16().double()  # rounded like the output
    err = float((y.double() - ref).norm() / ref.norm())
    assert err < 1e-3, err

    # the runner uses the merged weight after a refresh, and is back to the base output when it is removed
    r.refresh_weights()
    lora_out = r.forward(x, temb, None, None, meta, context=ctx).clone()
    assert not torch.equal(lora_out, base_out)
    weights.unmerge_lora(lin)
    assert lin._fp8_weight is base_w and lin._fp8_weight_scale is base_s
    r.refresh_weights()
    again = r.forward(x, temb, None, None, meta, context=ctx)
    assert torch.equal(again.view(torch.int16), base_out.view(torch.int16))
