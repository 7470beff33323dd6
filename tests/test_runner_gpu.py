"""The composed DiT block loop (H3FastRunner) on the GPU.

1. Sequence parallelism is exact: the block loop sharded over P ranks (emulated in one process, the same stages, buffers
   and all-to-all layouts as the NCCL path) gives bit-identical output to one rank, for P = 2 and 4, with full and
   48-row tiles. Every step is row-, tile- or (head, tile)-local, so nothing may change.
2. Each stage of a block is checked against the oracle on the stage's own GPU inputs (teacher forcing): quantized bytes
   against the restated quantizers (codes within the oracle's ambiguity windows), GEMMs against dequantize-then-matmul
   in fp32, tile scores and top-k selection bit-exact, FP8 attention within rel-Frobenius 2e-2 of exact attention over
   the same quantized operands.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle import vsa as ov
from test_oracle import assert_codes

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def deq_nvfp4(q: torch.Tensor, sf: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """NVFP4 codes x block scales (no global scale) -> fp32 [rows, K], plain torch on the GPU (test-side only)."""
    lut = torch.tensor(oq.E2M1_VALUES, device=q.device)
    codes = torch.stack([q[:rows] & 15, q[:rows] >> 4], -1).reshape(rows, K)
    vals = lut[codes.long()].view(rows, K // 16, 16)
    r = torch.arange(rows, device=q.device)[:, None]
    c = torch.arange(K // 16, device=q.device)[None, :]
    off = (r >> 7) * (K // 64) * 512 + (c >> 2) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3)
    s = sf.reshape(-1)[off].view(torch.float8_e4m3fn).float()
    return (vals * s[..., None]).reshape(rows, K)


def weight_fp32(fused: dict) -> torch.Tensor:
    """Dense fp32 [N, K] of a fused packed operand, global scales applied per column."""
    w = fused["w"]
    if fused["fmt"] == "nvfp4":
        d = deq_nvfp4(w, fused["sf"], w.shape[0], w.shape[1] * 2)
    else:
        d = w.float()
    return d * fused["col"][:, None]


def codes_of(h: torch.Tensor, K: int) -> np.ndarray:
    q = h.cpu().numpy()
    return np.stack([q & 15, q >> 4], -1).reshape(q.shape[0], K)


@pytest.fixture(scope="module")
def pkg(h3b):
    from fasth3_b200 import model, runner
    return model, runner


def make(pkg, blocks, fmt="nvfp4", grid=(7, 16, 16), seed=0):
    model, runner = pkg
    cfg = model.DiTConfig(blocks=blocks, fmt=fmt)
    m = model.DiTModel.random(cfg, device=DEV, seed=seed)
    T, Hh, Ww = grid
    g = torch.Generator(device=DEV).manual_seed(1000 + seed)
    x = torch.randn(1, T * Hh * Ww, cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    return m, x, ctx, temb, meta


@pytest.mark.parametrize("grid", [(8, 16, 16), (7, 16, 16)])
def test_sharded_block_loop_equals_single_rank(pkg, grid):
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=2, grid=grid)
    ref = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(ref.float()).all()
    assert rel(ref.float(), x.float()) > 1e-2  # the blocks did change the stream
    for P in (2, 4):
        got = runner.H3FastRunner(m, runner.VirtualSeqParallel(P)).forward(x, temb, None, None, meta, context=ctx)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), P


def make_prefixed(pkg, blocks, prefix=100, grid=(7, 16, 16), seed=3, **meta_kw):
    """A sequence of ``prefix`` exempt tokens ahead of a video latent, described by FastVideo-style metadata (the layout
    is built from untile_combined_index / variable_block_sizes), with RoPE tables in packed token order."""
    model, runner = pkg
    from fasth3_b200 import layout
    cfg = model.DiTConfig(blocks=blocks, fmt="nvfp4")
    m = model.DiTModel.random(cfg, device=DEV, seed=seed)
    md = layout.vsa_metadata(grid, prefix)
    S = md["untile_combined_index"].numel()
    T, Hh, Ww = grid
    tok = torch.arange(T * Hh * Ww)
    pos = torch.zeros(S, 3)
    pos[:prefix, 0] = torch.arange(prefix).float() * 0.25  # any fixed positions for the exempt tokens
    pos[prefix:] = torch.stack([tok // (Hh * Ww), (tok // Ww) % Hh, tok % Ww], 1).float()
    cos, sin = layout.rope_positions(pos)
    g = torch.Generator(device=DEV).manual_seed(2000 + seed)
    x = torch.randn(1, S, cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=None, untile_combined_index=md["untile_combined_index"],
                          variable_block_sizes=md["variable_block_sizes"], num_prefix_tiles=md["num_prefix_tiles"],
                          video_tile_spans=md["video_tile_spans"], **meta_kw)
    return m, x, ctx, temb, meta, (cos.to(DEV), sin.to(DEV))


def test_prefix_spans_and_dense_layers_drive_the_selection(pkg):
    """With prefix tiles, a video span at sparsity 0.75 and block 1 dense: every video query tile keeps the prefix
    tiles plus compute_topk(0.75, video tiles) of the span in sparse blocks and every tile in the dense block; prefix
    query tiles keep every tile. The sharded loop (layout from metadata) equals one rank bit for bit."""
    _, runner = pkg
    from fasth3_b200 import layout
    # 200 prefix tokens (4 tiles, the last one of 8 tokens) + 32 video tiles: 36 tiles, an even count per rank at P=2
    m, x, ctx, temb, meta, rot = make_prefixed(pkg, blocks=2, prefix=200, span_sparsities=[0.75], dense_layers=(1,))
    nums = {}
    r = runner.H3FastRunner(m)
    r.trace = lambda i, stage, rank, t: nums.__setitem__(i, t["num"].clone()) if stage == "select" else None
    ref = r.forward(x, temb, None, rot, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(ref.float()).all()
    n_pre = meta.num_prefix_tiles
    a, b = meta.video_tile_spans[0]
    k = layout.compute_topk(0.75, b - a)
    sparse, dense = nums[0].cpu(), nums[1].cpu()
    assert (sparse[:, :n_pre] == b).all() and (sparse[:, n_pre:b] == n_pre + k).all()
    assert (dense[:, :b] == b).all()
    got = runner.H3FastRunner(m, runner.VirtualSeqParallel(2)).forward(x, temb, None, rot, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("prefix", [100, 128])
def test_dense_prefix_pass_merged_by_lse_equals_one_pass(pkg, prefix):
    """The dense-prefix mode (prefix queries x every key and other queries x prefix keys as a separate dense pass of
    this library's attention kernel, the sparse pass on the span tiles only, joined by the log-sum-exp merge in the
    gate quantizer) against the same block with the prefix tiles inside every selection list: the same attention up
    to accumulation order. The merged attention is restated from the traced pieces and compared before quantization
    (5e-3); the NVFP4 attention codes agree within one quantization step (6e-2)."""
    _, runner = pkg
    m, x, ctx, temb, meta, rot = make_prefixed(pkg, blocks=1, prefix=prefix, span_sparsities=[0.75])
    cap = {}

    def tracer(tag):
        def t(i, stage, rank, ts):
            if stage == "gate":
                cap[(tag, i)] = (ts["a"].clone(), ts["a_sf"].clone(), ts["sa"].clone(), ts["ob"].clone())
            if stage == "dense_prefix":
                cap[("dense", i)] = {k: v.clone() for k, v in ts.items()}
        return t

    r1 = runner.H3FastRunner(m)
    r1.trace = tracer("one")
    out1 = r1.forward(x, temb, None, rot, meta, context=ctx)
    meta2 = runner.VsaMeta(**{**meta.__dict__, "dense_prefix": True})
    r2 = runner.H3FastRunner(m)
    r2.trace = tracer("split")
    out2 = r2.forward(x, temb, None, rot, meta2, context=ctx)
    torch.cuda.synchronize()
    rows = x.shape[1]
    slot = r2.layouts[next(iter(r2.layouts))][1][0].b["slot"].long()
    # one block: both runs see the same input (in deeper stacks the residual streams drift apart by the NVFP4
    # re-quantization of each block's attention output, and near-tie selections then differ)
    for i in range(1):
        a1, sf1, s1, ob1 = cap[("one", i)]
        a2, sf2, s2, _ = cap[("split", i)]
        # the merge the gate quantizer performs, restated in float64 from the traced pieces: the dense pass (o1,
        # natural-log LSEs) and the sparse pass (its output and log2 LSE; prefix rows take the dense pass alone)
        d = cap[("dense", i)]
        ob2 = _planes(d["ob_x"]).double()[:, slot].transpose(0, 1)  # [rows, H, 128]
        l1 = torch.cat([d["lse1a"], d["lse1b"]], 1).double().t() / math.log(2.0)  # [rows, H], log2
        l2 = d["lse2"].double()[:, slot].t()
        n1 = d["lse1a"].shape[1]
        l2[:n1] = -float("inf")
        m = torch.maximum(l1, l2)
        w1 = torch.where(torch.isfinite(m), torch.exp2(l1 - m), torch.zeros_like(m))
        w2 = torch.where(torch.isfinite(m), torch.exp2(l2 - m), torch.zeros_like(m))
        merged = (w1[..., None] * d["o1"].double() + torch.nan_to_num(w2[..., None] * ob2)) / (w1 + w2)[..., None]
        one = ob1.double()[:, slot].transpose(0, 1)
        assert rel(merged, one) < 5e-3, (i, rel(merged, one))
        # after the NVFP4 re-quantization of either, codes near a rounding boundary may differ by one step
        d1 = deq_nvfp4(a1, sf1, rows, a1.shape[1] * 2) * s1[:, None]
        d2 = deq_nvfp4(a2, sf2, rows, a2.shape[1] * 2) * s2[:, None]
        assert rel(d2, d1) < 6e-2, (i, rel(d2, d1))
    # the block output carries the re-quantization noise of two more NVFP4 stages (out-projection input, FFN
    # intermediate): a gross-error bound only; the merged attention above is the precise check
    assert rel(out2.float(), out1.float()) < 0.1


def test_f16_v_runner_equals_e4m3_v_runner(pkg):
    """The tile kernel's runner with V tiles as f16 (decoded once by the prologue) and with E4M3 V tiles (converted by
    the attention kernel): the same values reach the tensor cores, so the block loop's output is identical bit for bit,
    sharded too; the default runner (wide-step kernel) agrees with them."""
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=2, grid=(7, 16, 16))
    a = runner.H3FastRunner(m, v_f16=True, attn_kernel="tile").forward(x, temb, None, None, meta, context=ctx)
    b = runner.H3FastRunner(m, v_f16=False, attn_kernel="tile").forward(x, temb, None, None, meta, context=ctx)
    c = runner.H3FastRunner(m, runner.VirtualSeqParallel(2), v_f16=True, attn_kernel="tile").forward(
        x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert torch.equal(a.view(torch.int16), c.view(torch.int16))
    # the default runner (wide-step kernel: the tile kernel's two streams and merge, two key tiles per running-maximum
    # update) against the tile kernel's: block 0's attention output within 3e-3; the final output after two blocks of
    # NVFP4 re-quantization (a 4-bit code that flips moves its element by up to half) only within a gross bound
    attn = {}

    def keep(tag):
        return lambda i, stage, rank, t: attn.__setitem__(tag, t["ob_x"].float().clone()) if (i, stage) == (0, "attn") \
            else None

    rw, rt = runner.H3FastRunner(m), runner.H3FastRunner(m, v_f16=True, attn_kernel="tile")
    rw.trace, rt.trace = keep("wide"), keep("tile")
    w = rw.forward(x, temb, None, None, meta, context=ctx)
    t = rt.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.equal(t.view(torch.int16), a.view(torch.int16))
    assert float((attn["wide"] - attn["tile"]).norm() / attn["tile"].norm()) < 3e-3
    assert float((w.float() - a.float()).norm() / a.float().norm()) < 0.2


def test_balanced_tile_order(pkg):
    """tile_order="balanced" (the 48-row tiles of the 3-frame slab spread through the list): the sharded forward equals
    one rank's bit for bit; against the reference order, block 0's per-tile statistics and tile scores are the same
    values renumbered, every query tile selects the same key tiles, and the output differs only by the order in which
    each query tile's key tiles are accumulated (a gross bound after two blocks of NVFP4 re-quantization)."""
    _, runner = pkg
    from fasth3_b200 import layout
    m, x, ctx, temb, meta = make(pkg, blocks=2, grid=(7, 16, 16))
    rec = {}

    def keep(tag):
        def f(i, stage, rank, t):
            if i == 0 and stage in ("prologue", "select"):
                rec[(tag, stage)] = {k: v.clone() for k, v in t.items() if v is not None}
        return f

    rr, rb = runner.H3FastRunner(m), runner.H3FastRunner(m, tile_order="balanced")
    rr.trace, rb.trace = keep("ref"), keep("bal")
    ref = rr.forward(x, temb, None, None, meta, context=ctx)
    bal = rb.forward(x, temb, None, None, meta, context=ctx)
    for P in (2, 4):
        got = runner.H3FastRunner(m, runner.VirtualSeqParallel(P), tile_order="balanced").forward(
            x, temb, None, None, meta, context=ctx)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), bal.view(torch.int16)), P
    src = layout.balanced_order(layout.tile_layout(*meta.grid)).source.to(DEV)
    assert not torch.equal(src, torch.arange(src.numel(), device=DEV))
    pb, pr = rec[("bal", "prologue")], rec[("ref", "prologue")]
    for k in ("qs", "ks", "vs", "qp", "kp"):
        assert torch.equal(pb[k], pr[k][:, src]), k
    sb, sr = rec[("bal", "select")], rec[("ref", "select")]
    assert torch.equal(sb["sc"], sr["sc"][:, src][:, :, src])
    assert torch.equal(sb["num"], sr["num"][:, src])
    k = meta.topk
    assert bool((sb["num"] == k).all())
    chosen_bal = torch.sort(src[sb["idx"][:, :, :k].long()], -1).values
    chosen_ref = torch.sort(sr["idx"][:, src, :k].long(), -1).values
    assert torch.equal(chosen_bal, chosen_ref)
    assert float((bal.float() - ref.float()).norm() / ref.float().norm()) < 0.2
    # a layout from metadata keeps its prefix tiles first: no balanced order
    mp, xp, ctxp, tp, metap, rot = make_prefixed(pkg, blocks=1)
    with pytest.raises(ValueError, match="balanced"):
        runner.H3FastRunner(mp, tile_order="balanced").forward(xp, tp, None, rot, metap, context=ctxp)


def test_static_ffn_requant_runner(pkg):
    """ffn_requant="static": the first forward runs the per-row path (its output equals the default runner's bit for
    bit) and records each block's fixed FFN global scale; later forwards quantize fc_in's output in its epilogue under
    that scale. The result stays at the NVFP4 noise level of the per-row rule, and the sharded runner (the scale being
    the maximum over ranks) equals one rank bit for bit."""
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=2, grid=(7, 16, 16))
    ref = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    st = runner.H3FastRunner(m, ffn_requant="static")
    first = st.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int16), ref.view(torch.int16))
    assert bool((st.ffn_scales > 0).all())
    second = st.forward(x, temb, None, None, meta, context=ctx)
    sharded = runner.H3FastRunner(m, runner.VirtualSeqParallel(2), ffn_requant="static")
    sharded.forward(x, temb, None, None, meta, context=ctx)
    third = sharded.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.equal(sharded.ffn_scales, st.ffn_scales)
    assert torch.equal(third.view(torch.int16), second.view(torch.int16))
    # two NVFP4 quantizations of the FFN intermediate (per-row vs fixed global scale) differ by about sqrt(2) times
    # e2m1's relative noise (~0.09 each on this data), which is what the blocks' updates show
    upd_ref, upd = (ref.float() - x.float()), (second.float() - x.float())
    assert rel(upd, upd_ref) < 0.2, rel(upd, upd_ref)
    with pytest.raises(ValueError):
        runner.H3FastRunner(m, ffn_requant="per-tile")


def test_forward_raises_on_an_overlong_selection(pkg):
    """The attention kernel holds at most 1024 selected key tiles per query tile. A longer list is not a fault: the
    kernel clamps it and records H3B_EINVAL in its status word, and forward raises instead of returning the truncated
    attention. The read clears the word, so the next valid step returns normally."""
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=1, grid=(4, 64, 288))  # 1152 tiles of 64 tokens
    r = runner.H3FastRunner(m)
    meta.topk = 1100
    with pytest.raises(RuntimeError, match="EINVAL"):
        r.forward(x, temb, None, None, meta, context=ctx)
    meta.topk = 32
    out = r.forward(x, temb, None, None, meta, context=ctx)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("fmt", ["nvfp4", "fp8"])
def test_gate_compress_branch(pkg, fmt):
    """The optional gate-compress branch (gate GEMM and compressed attention on the side stream, joined in the gate
    quantizer): sharded equals single rank bit for bit (the compressed outputs take a heads -> sequence exchange), the
    gate GEMM matches dequantize-then-matmul, the compressed branch matches softmax(sc) @ vp, and the branch changes
    the block's output."""
    model, runner = pkg
    cfg = model.DiTConfig(blocks=1, fmt=fmt, gate_compress=True)
    m = model.DiTModel.random(cfg, device=DEV, seed=9)
    grid = (8, 16, 16)
    g = torch.Generator(device=DEV).manual_seed(77)
    x = torch.randn(1, grid[0] * grid[1] * grid[2], cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    r = runner.H3FastRunner(m)
    rec = {}

    def trace(i, stage, rank, tensors):
        if stage in ("select", "gate"):
            rec[stage] = {k: (v.clone() if v is not None else None) for k, v in tensors.items()}

    r.trace = trace
    ref = r.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    got = runner.H3FastRunner(m, runner.VirtualSeqParallel(2)).forward(x, temb, None, None, meta, context=ctx)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    # gate GEMM: g = h @ Wg^T without h's row scale (the gate quantizer applies it)
    t = rec["gate"]
    K = cfg.hidden
    rows = t["g"].shape[0]
    if fmt == "nvfp4":
        h = deq_nvfp4(t["h"], t["h_sf"], rows, K)
    else:
        h = t["h"].view(torch.float8_e4m3fn).float()
    want = (h.double() @ weight_fp32(r.fused[0]["gate"]).double().t()).bfloat16().double()
    assert rel(t["g"].double(), want) < 1e-3
    # compressed branch: oc = softmax(sc) @ vp, bf16
    sc, vp = rec["select"]["sc"].double(), rec["select"]["vp_all"].double()
    oc_want = torch.softmax(sc, -1) @ vp
    assert rel(t["oc"].double(), oc_want) < 4e-3
    # the branch contributes: the same model without it gives another output
    m.transformer_blocks[0].attn.to_gate_compress = None
    plain = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    assert not torch.equal(plain, ref)


def test_fp8_block_loop_runs_and_shards_exactly(pkg):
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=1, fmt="fp8", grid=(8, 16, 16))
    ref = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    got = runner.H3FastRunner(m, runner.VirtualSeqParallel(2)).forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(ref.float()).all()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


# ------------------------------------------------------------------------------------------------ stage parity
@pytest.fixture(scope="module")
def traced(pkg):
    _, runner = pkg
    m, x, ctx, temb, meta = make(pkg, blocks=1, grid=(7, 16, 16), seed=3)
    r = runner.H3FastRunner(m)
    rec = {}

    def trace(i, stage, rank, tensors):
        rec[(i, stage)] = {k: (v.clone() if v is not None else None) for k, v in tensors.items()}

    r.trace = trace
    out = r.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    full, states = r._layouts(meta, None)
    return {"rec": rec, "runner": r, "model": m, "tabs": m.adaln_tables(temb), "st": states[0], "full": full,
            "out": out, "ctx": ctx}


def _check_norm_fp4(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, h, h_sf, hs, eps, what):
    want = oq.resid_norm_quant(x.float().cpu().numpy(), shift=shift.float().cpu().numpy(),
                               scale=scale.float().cpu().numpy(), eps=eps, norm="layer", fp4=True)
    C = x.shape[1]
    assert_codes(codes_of(h, C), want["codes"], want["amb"], what)
    np.testing.assert_allclose(hs.cpu().numpy(), want["hs"], rtol=1e-6, err_msg=what)


def test_stage_norms(traced):
    rec, tabs, blk = traced["rec"], traced["tabs"], traced["model"].transformer_blocks[0]
    n1 = rec[(0, "norm1")]
    _check_norm_fp4(n1["x"], tabs[0, 0:1], tabs[0, 1:2], n1["h"], n1["h_sf"], n1["hs"], blk.eps, "norm1")
    n3 = rec[(0, "norm3")]
    _check_norm_fp4(rec[(0, "out_proj")]["x"], blk.norm3.shift, blk.norm3.scale, n3["h"], n3["h_sf"], n3["hs"],
                    blk.norm3.eps, "norm3")
    n2 = rec[(0, "norm2")]
    _check_norm_fp4(rec[(0, "cross_out")]["x"], tabs[0, 3:4], tabs[0, 4:5], n2["h"], n2["h_sf"], n2["hs"], blk.eps,
                    "norm2")


def upd_tol(x: torch.Tensor, upd: torch.Tensor) -> float:
    """Tolerance on a residual update read back as (x_new - x_old): 1e-2 plus the bf16 rounding of x_new (RMS relative
    error 2^-9/sqrt(3) of |x_new|) measured against |update|."""
    return 1e-2 + 2 * 1.2e-3 * float(x.norm() / upd.norm())


def test_stage_gemms(traced):
    rec, r, st, tabs = traced["rec"], traced["runner"], traced["st"], traced["tabs"]
    fz = r.fused[0]
    R, C, F = st.rows, r.hidden, r.ffn

    def a_of(stage, name="h", sf="h_sf"):
        return deq_nvfp4(rec[stage][name], rec[stage][sf], R, rec[stage][name].shape[1] * 2)

    # q/k/v: row scale deferred to the prologue
    want = a_of((0, "norm1")) @ weight_fp32(fz["qkv"]).t()
    assert rel(rec[(0, "qkv")]["qkv"].float(), want) < 3e-3
    # out-projection, gated residual in the epilogue
    g = rec[(0, "gate")]
    upd = tabs[0, 2].float() * (g["sa"][:, None] * (a_of((0, "gate"), "a", "a_sf") @ weight_fp32(fz["o"]).t()))
    x0 = rec[(0, "norm1")]["x"].float()
    x1 = rec[(0, "out_proj")]["x"].float()
    assert rel(x1, (x0 + upd).bfloat16().float()) < 1e-3
    assert rel(x1 - x0, upd) < upd_tol(x1, upd)
    # cross-attention query
    want = a_of((0, "norm3")) @ weight_fp32(fz["cq"]).t()
    assert rel(rec[(0, "cross_q")]["cq"].float(), want) < 3e-3
    # cross-attention output projection (ungated residual)
    ca = rec[(0, "cross_attn")]
    upd = ca["sa"][:, None] * (a_of((0, "cross_attn"), "a", "a_sf") @ weight_fp32(fz["co"]).t())
    x2 = rec[(0, "cross_out")]["x"].float()
    assert rel(x2, (x1 + upd).bfloat16().float()) < 1e-3
    # fc_in with GELU-tanh, then fc_out with the gated residual
    n2 = rec[(0, "norm2")]
    pre = n2["hs"][:, None] * (a_of((0, "norm2")) @ weight_fp32(fz["fc_in"]).t())
    want = torch.nn.functional.gelu(pre, approximate="tanh")
    mid = rec[(0, "ffn_mid")]
    assert rel(mid["u"].float(), want) < 3e-3
    upd = tabs[0, 5].float() * (mid["fs"][:, None] * (deq_nvfp4(mid["f"], mid["f_sf"], R, F) @
                                                      weight_fp32(fz["fc_out"]).t()))
    x3 = rec[(0, "fc_out")]["x"].float()
    assert rel(x3, (x2 + upd).bfloat16().float()) < 1e-3
    assert rel(x3 - x2, upd) < upd_tol(x3, upd)


def test_stage_ffn_requant(traced):
    mid = traced["rec"][(0, "ffn_mid")]
    u = mid["u"].float().cpu().numpy()
    am = np.abs(u).max(axis=1).astype(np.float32)
    s = np.maximum((am / oq.FP4_RANGE).astype(np.float32), oq.FP4_MIN_SCALE).astype(np.float32)
    codes, bits, amb, sf_amb = oq.nvfp4_blocks(u, (np.float32(1.0) / s).astype(np.float32))
    assert_codes(codes_of(mid["f"], u.shape[1]), codes, amb, "ffn requant")
    np.testing.assert_allclose(mid["fs"].cpu().numpy(), s, rtol=1e-6)


def test_stage_prologue_and_selection(traced):
    rec, r, st, blk = traced["rec"], traced["runner"], traced["st"], traced["model"].transformer_blocks[0]
    H, C = r.heads, r.hidden
    b = st.b
    qkv = rec[(0, "qkv")]["qkv"].float().cpu().numpy()
    hs = rec[(0, "norm1")]["hs"].cpu().numpy()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    want = ov.qkv_prologue8(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], hs, b["tile_row0"].cpu().numpy(),
                            b["vbs"].cpu().numpy(), f(blk.attn.norm_q.weight), f(blk.attn.norm_k.weight), f(b["cos"]),
                            f(b["sin"]), H, 1.0, 1.0, eps=blk.attn.norm_q.eps)
    p = rec[(0, "prologue")]
    vbs = b["vbs"].cpu().numpy()
    row0 = b["tile_row0"].cpu().numpy()
    for name, vals, sname in (("qb", want["q"], "qs"), ("kb", want["k"], "ks"), ("vb", want["v"], "vs")):
        got_s = p[sname].cpu().numpy()
        got_b = p[name].cpu().numpy()
        ok = total = 0
        for t in range(st.n_local):
            rows = vals[row0[t]:row0[t] + vbs[t]]  # [n, H, 128]
            am = np.abs(rows).max(axis=(0, 2)).astype(np.float32)
            np.testing.assert_allclose(got_s[:, t], np.maximum(am / 448.0, 1e-30), rtol=1e-2, err_msg=name)
            for h in range(H):
                w = oq.e4m3_decode(oq.e4m3_encode(rows[:, h] / got_s[h, t]))
                g = _values(got_b[h, t * 64:t * 64 + vbs[t]])
                close = np.abs(g - w) <= np.maximum(np.abs(w), 2 ** -6) * 0.126
                ok += int(close.sum())
                total += close.size
        assert ok / total > 0.999, (name, ok / total)
    # tile means of the bf16 values
    for name, vals in (("qp", want["q"]), ("kp", want["k"])):
        got = p[name].cpu().numpy()
        for t in range(st.n_local):
            m = vals[row0[t]:row0[t] + vbs[t]].mean(axis=0)  # [H, 128]
            np.testing.assert_allclose(got[:, t], m, rtol=5e-2, atol=2e-2, err_msg=name)
    # scores bit-exact, selection bit-exact (ties to the lowest column)
    s = rec[(0, "select")]
    n = st.n_local
    sc = ov.tile_scores(s["qp_all"].cpu().numpy(), s["kp_all"].cpu().numpy(), 1.0 / math.sqrt(128))
    np.testing.assert_array_equal(s["sc"].cpu().numpy(), sc)
    idx, num = ov.topk_rows(sc, n, n, 0, [(0, n, 8)], False)
    num_g = s["num"].cpu().numpy()
    np.testing.assert_array_equal(num_g, num)
    idx_g = s["idx"].cpu().numpy()
    for h in range(H):
        for t in range(n):
            np.testing.assert_array_equal(idx_g[h, t, :num[h, t]], idx[h, t, :num[h, t]])
    np.testing.assert_array_equal(s["vs_head"].cpu().numpy(), s["vs_all"].cpu().numpy().max(axis=1))


def _values(t) -> np.ndarray:
    """E4M3 codes (uint8) or the f16 tensors holding their values (the f16-V path) -> float32 values."""
    t = t.cpu() if isinstance(t, torch.Tensor) else torch.from_numpy(t)
    return t.float().numpy() if t.dtype == torch.float16 else oq.e4m3_decode(t.numpy())


def _planes(x: torch.Tensor) -> torch.Tensor:
    """A one-rank runner's head-sharded buffer [G=1, P=1, H, rows, 128] as [H, rows, 128]."""
    return x.reshape(-1, *x.shape[-2:])


def _deq_tiles(codes: torch.Tensor, scales: torch.Tensor) -> np.ndarray:
    """E4M3 [H, n*64, 128] (codes, or f16 values) with per-(head, tile) scales [H, n] -> float32."""
    H, rows_pad, D = codes.shape
    v = _values(codes).reshape(H, rows_pad // 64, 64, D)
    return (v * scales.cpu().numpy()[:, :, None, None]).reshape(H, rows_pad, D)


def test_stage_self_attention(traced):
    rec, st = traced["rec"], traced["st"]
    s, a = rec[(0, "select")], rec[(0, "attn")]
    q = _deq_tiles(_planes(s["qb_x"]), s["qs_all"])
    k = _deq_tiles(_planes(s["kb_x"]), s["ks_all"])
    v = _deq_tiles(_planes(s["vb_x"]), s["vs_all"])
    vbs = st.b["vbs"].cpu().numpy()
    want = ov.vsa_fine(q, k, v, s["idx"].cpu().numpy(), s["num"].cpu().numpy(), vbs, 1.0 / math.sqrt(128))
    got = _planes(a["ob_x"]).float().cpu().numpy()
    mask = (np.arange(got.shape[1]) % 64)[None, :] < np.repeat(vbs, 64)[None, :]
    g, w = got[:, mask[0]], want[:, mask[0]]
    err = np.linalg.norm(g - w) / np.linalg.norm(w)
    assert err < 2e-2, err
    # attention output -> compact rows, NVFP4 row quantization
    gt = rec[(0, "gate")]
    ref = ov.attn_gate_quant(gt["ob"].float().cpu().numpy(), st.b["slot"].cpu().numpy(), st.rows, fp4=True)
    assert_codes(codes_of(gt["a"], ref["codes"].shape[1]), ref["codes"], ref["amb"], "attn out quant")
    np.testing.assert_allclose(gt["sa"].cpu().numpy(), ref["s"], rtol=1e-6)


def test_stage_cross_attention(traced):
    rec, r, st, blk = traced["rec"], traced["runner"], traced["st"], traced["model"].transformer_blocks[0]
    H, C = r.heads, r.hidden
    txt = rec[(0, "text")]
    fz = r.fused[0]
    L = txt["kv"].shape[0]
    # text K/V projection (row scale deferred), per-head RMSNorm for K, per-tile E4M3
    a = deq_nvfp4(txt["tq"], txt["tsf"], L, txt["tq"].shape[1] * 2)
    want = a @ weight_fp32(fz["ckv"]).t()
    assert rel(txt["kv"].float(), want) < 3e-3
    kv = txt["kv"].float() * txt["ts"][:, None]
    kf = kv[:, :C].view(L, H, 128)
    kf = kf * torch.rsqrt(kf.pow(2).mean(-1, keepdim=True) + blk.attn2.norm_k.eps) * blk.attn2.norm_k.weight.float()
    vf = kv[:, C:].view(L, H, 128)
    k_deq = torch.from_numpy(_deq_tiles(txt["kb"], txt["ks"])).to(DEV)
    v_deq = torch.from_numpy(_deq_tiles(txt["vb"], txt["vs"])).to(DEV)
    assert rel(k_deq, kf.permute(1, 0, 2)) < 4e-2
    assert rel(v_deq, vf.permute(1, 0, 2)) < 4e-2
    # cross queries: RMSNorm of (cq * hs), per-tile E4M3
    cq = rec[(0, "cross_q")]
    hs = rec[(0, "norm3")]["hs"]
    qf = (cq["cq"].float() * hs[:, None]).view(st.rows, H, 128)
    qf = qf * torch.rsqrt(qf.pow(2).mean(-1, keepdim=True) + blk.attn2.norm_q.eps) * blk.attn2.norm_q.weight.float()
    q_deq = torch.from_numpy(_deq_tiles(cq["cqb"], cq["cqs"])).to(DEV)
    slot = st.b["slot"].long()
    assert rel(q_deq[:, slot], qf.permute(1, 0, 2)) < 4e-2
    # dense attention over the 512 text keys with the same quantized operands
    p = torch.softmax((q_deq.double() @ k_deq.double().transpose(1, 2)) / math.sqrt(128), -1)
    want = (p @ v_deq.double()).float()
    got = rec[(0, "cross_attn")]["cob"].float()
    assert rel(got[:, slot], want[:, slot]) < 2e-2


# ------------------------------------------------------------------------------------------------ config 3 chain
def test_fp8_block_chain_stages(pkg):
    """BASELINE config 3's chain at 1000 rows, each stage against the oracle on its own GPU inputs."""
    _, runner = pkg
    chain = runner.Fp8BlockChain.random(DEV, seed=5)
    g = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(1000, 5120, device=DEV, generator=g).bfloat16()
    tabs = (torch.randn(6, 5120, device=DEV, generator=g) * 0.1).bfloat16()
    rec = {}
    chain.trace = lambda stage, t: rec.__setitem__(stage, {k: v.clone() for k, v in t.items()})
    x0 = x.clone()
    chain(x, tabs)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    # LayerNorm + modulate + FP8 (attention half)
    want = oq.resid_norm_quant(f(x0), shift=f(tabs[0:1]), scale=f(tabs[1:2]), eps=1e-6, norm="layer")
    assert_codes(rec["norm1"]["h"].view(torch.uint8).cpu().numpy(), want["h"], want["amb"], "chain norm1")
    # QKV GEMM with row and channel scales, then FP8 of the V third
    h = rec["norm1"]["h"].float() * rec["norm1"]["hs"][:, None]
    qkv_ref = h @ weight_fp32(chain.qkv).t()
    assert rel(rec["qkv"]["qkv"].float(), qkv_ref) < 3e-3
    codes, s, amb = oq.quant_fp8_rows(f(rec["qkv"]["qkv"][:, 2 * 5120:]))
    assert_codes(rec["qkv"]["a"].view(torch.uint8).cpu().numpy(), codes, amb, "chain V quant")
    # out-projection with the gated residual
    a = rec["qkv"]["a"].float() * rec["qkv"]["sa"][:, None]
    upd = tabs[2].float() * (a @ weight_fp32(chain.o).t())
    x1 = rec["out_proj"]["x"].float()
    assert rel(x1, (x0.float() + upd).bfloat16().float()) < 1e-3
    # second norm, fc_in with GELU-tanh, FP8 of the intermediate, fc_out with the gated residual
    want = oq.resid_norm_quant(f(rec["out_proj"]["x"]), shift=f(tabs[3:4]), scale=f(tabs[4:5]), eps=1e-6,
                               norm="layer")
    assert_codes(rec["norm2"]["h"].view(torch.uint8).cpu().numpy(), want["h"], want["amb"], "chain norm2")
    h2 = rec["norm2"]["h"].float() * rec["norm2"]["hs"][:, None]
    u_ref = torch.nn.functional.gelu(h2 @ weight_fp32(chain.fc_in).t(), approximate="tanh")
    assert rel(rec["ffn_mid"]["u"].float(), u_ref) < 3e-3
    codes, s, amb = oq.quant_fp8_rows(f(rec["ffn_mid"]["u"]))
    assert_codes(rec["ffn_mid"]["f"].view(torch.uint8).cpu().numpy(), codes, amb, "chain FFN quant")
    fq = rec["ffn_mid"]["f"].float() * rec["ffn_mid"]["fs"][:, None]
    upd = tabs[5].float() * (fq @ weight_fp32(chain.fc_out).t())
    assert rel(rec["fc_out"]["x"].float(), (x1 + upd).bfloat16().float()) < 1e-3


@pytest.mark.parametrize("gate", [False, True])
def test_graphed_forward_replays_the_eager_result(pkg, gate):
    """The CUDA-graph replay of the block loop gives the eager forward's bytes, for new inputs copied into the graph
    (and with the side-stream gate-compress branch inside the graph)."""
    model, runner = pkg
    cfg = model.DiTConfig(blocks=2, gate_compress=gate)
    m = model.DiTModel.random(cfg, device=DEV, seed=14)
    grid = (8, 16, 16)
    g = torch.Generator(device=DEV).manual_seed(90)
    S = grid[0] * grid[1] * grid[2]
    xs = [torch.randn(1, S, cfg.hidden, device=DEV, generator=g).bfloat16() for _ in range(2)]
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    r = runner.H3FastRunner(m)
    gf = runner.GraphedForward(r, xs[0], temb, meta, ctx)
    for x in (xs[1], xs[0]):
        got = gf(x, temb).clone()
        want = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
