"""INT8 QK^T in the block-sparse attention (tcgen05 kind::i8, exact s32 scores): parity with exact attention over the
same int8 Q/K and E4M3 V, the accuracy gain over E4M3 Q/K against attention on the unquantized inputs, and the
prologue's int8 variant against its E4M3 form on the same inputs."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from cases import prologue_inputs
from oracle import quant as oq
from oracle import vsa as ov

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _quant_tiles(x: torch.Tensor, n: int, int8: bool):
    """Per (head, 64-row tile) symmetric quantization of x [heads, n*64, 128]: (codes uint8 view, scales [heads, n],
    dequantized float64)."""
    heads = x.shape[0]
    t = x.float().view(heads, n, 64, 128)
    amax = t.abs().amax(dim=(2, 3))
    if int8:
        s = (amax / 127.0).clamp(min=1e-30)
        c = torch.round(t / s[:, :, None, None]).clamp(-127, 127).to(torch.int8)
        return c.view(torch.uint8).reshape(heads, n * 64, 128), s, c.double() * s.double()[:, :, None, None]
    s = (amax / 448.0).clamp(min=1e-30)
    c = torch.from_numpy(oq.e4m3_encode((t / s[:, :, None, None]).numpy()))
    deq = torch.from_numpy(oq.e4m3_decode(c.numpy())).double() * s.double()[:, :, None, None]
    return c.reshape(heads, n * 64, 128), s, deq


def _case(heads=2, n=24, k=6, seed=70):
    g = torch.Generator().manual_seed(seed)
    q, kk, v = (torch.randn(heads, n * 64, 128, generator=g).bfloat16() for _ in range(3))
    idx = torch.stack([torch.randperm(n, generator=g)[:k].sort().values for _ in range(heads * n)])
    return q, kk, v, idx.view(1, heads, n, k).to(torch.int32), torch.full((1, heads, n), k, dtype=torch.int32)


def _run(ops, q, kk, v, idx, num, int8: bool):
    heads, rows, _ = q.shape
    n = rows // 64
    qc, qs, qd = _quant_tiles(q, n, int8)
    kc, ks, kd = _quant_tiles(kk, n, int8)
    vc, vs, vd = _quant_tiles(v, n, False)
    vbs = torch.full((n,), 64, dtype=torch.int32)
    out = torch.zeros(heads, rows, 128, device=DEV, dtype=torch.bfloat16)
    dv = lambda t: t.contiguous().to(DEV)  # noqa: E731
    sm = 1.0 / math.sqrt(128)
    ops.vsa_fp8_ex(dv(qc), dv(kc), dv(vc), out, dv(idx), dv(num), dv(vbs), dv(vbs), dv(vs), dv(vs.amax(1)),
                   sm * math.log2(math.e), heads, n, n, rows, rows, qs=dv(qs), ks=dv(ks), idx_ld=idx.shape[-1],
                   qk_int8=int8)
    torch.cuda.synchronize()
    assert ops.vsa_status(reset=True) == 0
    view = lambda t: t.reshape(heads, rows, 128).numpy()  # noqa: E731
    ref_q = ov.vsa_fine(view(qd), view(kd), view(vd), idx.numpy()[0], num.numpy()[0], vbs.numpy(), sm)
    exact = ov.vsa_fine(q.double().numpy(), kk.double().numpy(), v.double().numpy(), idx.numpy()[0], num.numpy()[0],
                        vbs.numpy(), sm)
    return out.cpu().double().numpy(), ref_q, exact


def test_int8_qk_attention_matches_exact_over_its_operands(ops):
    q, kk, v, idx, num = _case()
    got, ref, _ = _run(ops, q, kk, v, idx, num, int8=True)
    assert _rel(got, ref) < 1e-2  # the E4M3 path's bar (f16 P, ~2^-9)


def test_int8_qk_is_more_accurate_than_e4m3(ops):
    q, kk, v, idx, num = _case(seed=71)
    got8, _, exact = _run(ops, q, kk, v, idx, num, int8=True)
    gotf, _, _ = _run(ops, q, kk, v, idx, num, int8=False)
    e8, ef = _rel(got8, exact), _rel(gotf, exact)
    assert e8 < ef, (e8, ef)


def test_prologue_int8_variant_against_e4m3_form(ops):
    heads, n_tiles = 3, 10
    d = {k: t.to(DEV) for k, t in prologue_inputs(heads, n_tiles, 73).items()}
    n_ext = n_tiles
    rows_pad = n_ext * 64
    res = {}
    for int8 in (False, True):
        z = lambda *sh, dt=torch.uint8: torch.zeros(*sh, device=DEV, dtype=dt)  # noqa: E731
        qb, kb, vb = z(heads, rows_pad, 128), z(heads, rows_pad, 128), z(heads, rows_pad, 128)
        qs, ks, vs = (torch.ones(heads, n_ext, device=DEV) for _ in range(3))
        vs_head = torch.zeros(heads, device=DEV)
        qp, kp, vp = (z(heads, n_tiles, 128, dt=torch.float32) for _ in range(3))
        ops.qkv_prologue8(d["q"], d["k"], d["v"], d["s1"], d["tile_row0"], d["vbs"], d["wq"], d["wk"], d["cos"],
                          d["sin"], 1.0, 1.0, qb, kb, vb, vs, vs_head, qp, kp, vp, heads, n_tiles, 64, 1e-5,
                          qs_blk=qs, ks_blk=ks, qk_int8=int8)
        torch.cuda.synchronize()
        res[int8] = {k: t.cpu() for k, t in dict(qb=qb, kb=kb, vb=vb, qs=qs, ks=ks, vs=vs, vs_head=vs_head, qp=qp,
                                                  kp=kp, vp=vp).items()}
    e, i = res[False], res[True]
    for key in ("vb", "vs", "vs_head", "qp", "kp", "vp"):  # V and the means do not depend on the Q/K code
        assert torch.equal(e[key].view(torch.uint8), i[key].view(torch.uint8)), key
    for c, s in (("qb", "qs"), ("kb", "ks")):
        # same tile amax: the scales differ by 448/127 up to one rounding
        np.testing.assert_allclose(i[s].numpy(), e[s].numpy() * (448.0 / 127.0), rtol=1e-6)
        s8 = i[s].numpy().repeat(64, 1)[:, :, None]
        se = e[s].numpy().repeat(64, 1)[:, :, None]
        x8 = i[c].view(torch.int8).numpy().astype(np.float64) * s8
        xe = oq.e4m3_decode(e[c].numpy()).astype(np.float64) * se
        # both within their rounding of the same bf16 values: half an int8 step plus one E4M3 relative step
        assert (np.abs(x8 - xe) <= 0.51 * s8 + np.abs(xe) * 2.0 ** -3 + 1e-12).all(), c
        assert np.abs(i[c].view(torch.int8).numpy()).max() == 127


def test_runner_with_int8_qk(h3b):
    """The block loop with INT8 QK^T: sharded equals single rank bit for bit, and the output stays close to the E4M3
    run (both approximate the same attention)."""
    model, runner = h3b.model, h3b.runner
    cfg = model.DiTConfig(blocks=1)
    m = model.DiTModel.random(cfg, DEV, seed=12)
    grid = (8, 16, 16)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(1, grid[0] * grid[1] * grid[2], cfg.hidden, device=DEV, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = runner.VsaMeta(grid=grid, topk=8)
    got = runner.H3FastRunner(m, qk_int8=True).forward(x, temb, None, None, meta, context=ctx)
    sharded = runner.H3FastRunner(m, runner.VirtualSeqParallel(2), qk_int8=True).forward(x, temb, None, None, meta,
                                                                                           context=ctx)
    e4 = runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    assert torch.equal(sharded.view(torch.int16), got.view(torch.int16))
    assert not torch.equal(got, e4)
    assert _rel(got.double().cpu().numpy(), e4.double().cpu().numpy()) < 5e-2
