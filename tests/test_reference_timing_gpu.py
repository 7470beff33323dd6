"""The reference's own kernels, built from its sources for sm_100a (``oracle/_ref``), timed beside this library's on
the same inputs and the same B200 -- the timing bar for each kernel. Outputs are compared too (bit for bit where the
kernels are bit-exact, within tolerance for the attention), so the two sides are known to do the same work.

Kernels (reference file:line -> this library):
  resid_norm_quant<5120, branch, RMS, FP8 | NVFP4>  h3fast.cu:188-265      -> h3b_resid_norm_quant
  qkv_prologue8 (40 heads, static Q/K scales)       h3fast.cu:376-510      -> h3b_qkv_prologue8
  topk_rows (top-32 of 512 and of 2016 tiles)       h3fast.cu:524-588      -> h3b_topk_rows
  attn_gate_quant<5120, FP8>                        h3fast.cu:688-741      -> h3b_attn_gate_quant
  VSA forward: the reference's BF16 kernel           vsa_bf16.cuh:197-1131  -> h3b_vsa_fp8 (E4M3 Q/K/V), h3b_vsa_fp8_ws
               (h3attn16.cu, built with VSA_LDRED off: tcgen05.ld.red is sm_103a-only)

Prints one line per kernel (``-s`` shows them): median milliseconds of 10 launches after 3 warm-ups (CUDA events) for
each side and the algorithmic GB/s or TFLOP/s. Nothing is asserted about speed.
"""
from __future__ import annotations

import json
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref():
    from oracle.ref_build.build_ref import load
    mod, cdll = load()
    if mod is None:
        pytest.skip("oracle/_ref/h3ref.so not present (built only where the reference sources are)")
    return mod, cdll


def _ref_attn():
    from oracle.ref_build.build_ref import load_attn16
    mod = load_attn16()
    if mod is None:
        pytest.skip("oracle/_ref/attn16/h3ref_attn16.so not present")
    return mod


def _time(fn, reps: int = 10) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    return ts[len(ts) // 2]


def _report(name: str, ref_ms: float, ours_ms: float, work: float, unit: str) -> None:
    scale = 1e9 if unit == "GB/s" else 1e12
    print("\n" + json.dumps({"kernel": name, "reference_ms": round(ref_ms, 4), "h3b_ms": round(ours_ms, 4),
                             "speedup": round(ref_ms / ours_ms, 3), "unit": unit,
                             "reference": round(work / (ref_ms * 1e-3) / scale, 1),
                             "h3b": round(work / (ours_ms * 1e-3) / scale, 1)}))


@pytest.mark.parametrize("fp4", [False, True])
def test_resid_norm_quant_timing(ops, fp4):
    _, cdll = _ref()
    C, rows = 5120, 32760
    g = torch.Generator(device=DEV).manual_seed(1)
    x = (torch.randn(rows, C, device=DEV, generator=g) * 3).bfloat16()
    y = torch.randn(rows, C, device=DEV, generator=g).bfloat16()
    sy = torch.rand(rows, device=DEV, generator=g) + 0.5
    tabs = (torch.randn(6, 3 * C, device=DEV, generator=g) * 0.3).bfloat16()
    idx = torch.randint(0, 6, (rows,), device=DEV, generator=g, dtype=torch.int32)
    nw = torch.randn(C, device=DEV, generator=g).bfloat16()
    shift, scale, gate = tabs[:, :C], tabs[:, C:2 * C], tabs[:, 2 * C:]
    hb = C // 2 if fp4 else C
    outs = [(torch.empty_like(x), torch.zeros(rows, hb, device=DEV, dtype=torch.uint8),
             torch.zeros(ops.sf_rows(rows), C // 16, device=DEV, dtype=torch.uint8) if fp4 else None,
             torch.zeros(rows, device=DEV)) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream
    P = lambda t: None if t is None else t.data_ptr()  # noqa: E731

    def ref():
        xo, h, hsf, hs = outs[0]
        assert cdll.h3ref_resid_norm_quant_5120(P(x), P(y), P(sy), P(gate), gate.stride(0), P(idx), P(nw), P(shift),
                                                P(scale), scale.stride(0), P(xo), P(h), P(hsf), P(hs), 1e-5, rows,
                                                st) == 0

    def ours():
        xo, h, hsf, hs = outs[1]
        ops.resid_norm_quant(x, y, sy, gate, idx, nw, shift, scale, xo, h, hsf, hs, 1e-5, norm="rms")

    t_ref, t_ours = _time(ref), _time(ours)
    for a, b in zip(outs[0], outs[1]):
        if a is not None:
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    byt = rows * C * 2 * 3 + rows * (hb + (C // 16 if fp4 else 0)) + rows * 4
    _report(f"resid_norm_quant<5120, branch, RMS, {'NVFP4' if fp4 else 'FP8'}> 32760 rows", t_ref, t_ours, byt, "GB/s")


def test_qkv_prologue8_timing(ops):
    mod, _ = _ref()
    heads, n_tiles = 40, 512
    rows, W = n_tiles * 64, heads * 128
    g = torch.Generator(device=DEV).manual_seed(2)
    q, k, v = (torch.randn(rows, W, device=DEV, generator=g).bfloat16() for _ in range(3))
    s1 = torch.rand(rows, device=DEV, generator=g) + 0.5
    wq, wk = (torch.randn(128, device=DEV, generator=g).bfloat16() for _ in range(2))
    ang = torch.rand(rows, 48, device=DEV, generator=g) * 6.28
    cos, sin = torch.cat([ang.cos()] * 2, -1).bfloat16(), torch.cat([ang.sin()] * 2, -1).bfloat16()
    vbs = torch.full((n_tiles,), 64, device=DEV, dtype=torch.int32)
    row0 = (torch.arange(n_tiles, device=DEV, dtype=torch.int32) * 64)
    inv_sq = inv_sk = 448.0 / math.sqrt(128)

    def bufs():
        z = lambda *sh, dt=torch.uint8: torch.zeros(*sh, device=DEV, dtype=dt)  # noqa: E731
        return [z(1, heads, rows, 128), z(1, heads, rows, 128), z(1, heads, rows, 128),
                torch.ones(heads, n_tiles, device=DEV), torch.zeros(heads, device=DEV),
                z(heads, n_tiles, 128, dt=torch.float32), z(heads, n_tiles, 128, dt=torch.float32),
                z(heads, n_tiles, 128, dt=torch.float32)]
    rb, ob = bufs(), bufs()

    def ref():
        mod.qkv_prologue8(q, k, v, s1, row0, vbs, wq, wk, cos, sin, inv_sq, inv_sk, *rb, heads, n_tiles, 64, 1e-5,
                          None, None, None)

    def ours():
        ops.qkv_prologue8(q, k, v, s1, row0, vbs, wq, wk, cos, sin, inv_sq, inv_sk, *ob, heads, n_tiles, 64, 1e-5)

    t_ref, t_ours = _time(ref), _time(ours)
    for a, b in zip(rb, ob):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    byt = 3 * rows * W * 2 + 3 * rows * W + 3 * heads * n_tiles * 128 * 4
    _report("qkv_prologue8 40 heads x 32768 rows", t_ref, t_ours, byt, "GB/s")


@pytest.mark.parametrize("n", [512, 2016])
def test_topk_rows_timing(ops, n):
    mod, _ = _ref()
    heads, k = 40, 32
    g = torch.Generator(device=DEV).manual_seed(3)
    sc = torch.randn(heads, n, n, device=DEV, generator=g)
    res = [(torch.full((1, heads, n, n), -1, device=DEV, dtype=torch.int32),
            torch.zeros(1, heads, n, device=DEV, dtype=torch.int32)) for _ in range(2)]

    def ref():
        mod.topk_rows(sc, n, n, 0, [0], [n], [k], res[0][0], res[0][1], False)

    def ours():
        ops.topk_rows(sc, n, n, 0, [0], [n], [k], res[1][0], res[1][1], False)

    t_ref, t_ours = _time(ref), _time(ours)
    assert torch.equal(res[0][1], res[1][1])
    assert torch.equal(res[0][0][..., :k], res[1][0][..., :k])
    _report(f"topk_rows top-{k} of {n} tiles, 40 heads", t_ref, t_ours, heads * n * n * 4 + heads * n * k * 4, "GB/s")


def test_attn_gate_quant_timing(ops):
    _, cdll = _ref()
    heads, n_tiles = 40, 512
    rows, W = n_tiles * 64, heads * 128
    g = torch.Generator(device=DEV).manual_seed(4)
    obuf = torch.randn(1, heads, rows, 128, device=DEV, generator=g).bfloat16()
    slot = torch.arange(rows, device=DEV, dtype=torch.int32)
    outs = [(torch.zeros(rows, W, device=DEV, dtype=torch.uint8), torch.zeros(rows, device=DEV)) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream

    def ref():
        assert cdll.h3ref_attn_gate_quant_5120(obuf.data_ptr(), None, None, None, slot.data_ptr(), rows, n_tiles, 64,
                                               outs[0][0].data_ptr(), None, outs[0][1].data_ptr(), rows, st) == 0

    def ours():
        ops.attn_gate_quant(obuf, None, None, None, slot, n_tiles, 64, outs[1][0].view(torch.float8_e4m3fn), None,
                            outs[1][1], rows)

    t_ref, t_ours = _time(ref), _time(ours)
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32))
    _report("attn_gate_quant<5120, FP8> 32768 rows", t_ref, t_ours, rows * W * 3 + rows * 4, "GB/s")


def test_vsa_attention_timing_config4(ops):
    """40 heads, 32768 tokens on an 8x64x64 grid (512 tiles of 64), top-32 key tiles per query
    tile. The reference's BF16 kernel reads bf16 Q/K/V in tile order; this library's reads the per-tile E4M3 codes of
    the same tensors. Same selection for both."""
    attn = _ref_attn()
    H, T, Hh, Ww, D, k = 40, 8, 64, 64, 128, 32
    S = T * Hh * Ww
    n = S // 64
    g = torch.Generator(device=DEV).manual_seed(11)
    q, kk, v = (torch.randn(H, S, D, device=DEV, generator=g).bfloat16() for _ in range(3))
    grid = torch.arange(S, device=DEV).view(T // 4, 4, Hh // 4, 4, Ww // 4, 4)
    perm = grid.permute(0, 2, 4, 1, 3, 5).reshape(-1).to(torch.int32)
    vbs = torch.full((n,), 64, device=DEV, dtype=torch.int32)
    row0 = (torch.arange(n, device=DEV) * 64).to(torch.int32)
    qb, kb = (torch.empty(H, S, D, device=DEV, dtype=torch.uint8) for _ in range(2))
    vb = torch.empty(H, S, D, device=DEV, dtype=torch.float16)  # this library's f16-V form
    qs, ks, vs = (torch.empty(H, n, device=DEV) for _ in range(3))
    vs_head = torch.zeros(H, device=DEV)
    qp, kp, vp = (torch.empty(H, n, D, device=DEV) for _ in range(3))
    ops.vsa_tile_quant(q, kk, v, perm, row0, vbs, qb, kb, vb, qs, ks, vs, qp, kp, vp, n, vs_head=vs_head)
    sc = torch.empty(H, n, n, device=DEV)
    sm_scale = 1.0 / math.sqrt(D)
    ops.tile_scores(qp, kp, sc, sm_scale)
    idx = torch.empty(1, H, n, n, device=DEV, dtype=torch.int32)
    num = torch.zeros(1, H, n, device=DEV, dtype=torch.int32)
    ops.topk_rows(sc, n, n, 0, [0], [n], [k], idx, num, False)
    out = torch.empty(1, H, S, D, device=DEV, dtype=torch.bfloat16)
    pl = perm.long()
    qt, kt, vt = (t[:, pl].unsqueeze(0).contiguous() for t in (q, kk, v))  # tile order, [1, H, S, D]
    q2k_idx = idx[0, :, :, :k].reshape(H * n, k).contiguous()
    q2k_num = num.reshape(-1).contiguous()

    def ref():
        return attn.vsa_bf16(qt, kt, vt, None, q2k_idx, q2k_num, vbs, sm_scale, False)[0]

    def ours():
        ops.vsa_fp8(qb, kb, vb, idx, num, vbs, sm_scale * math.log2(math.e), vs, vs_head, q_scale_blk=qs,
                    k_scale_blk=ks, out=out)

    def ours_wide():  # the runner's kernel: h3b_vsa_fp8_ws
        ops.vsa_fp8_ex(qb, kb, vb, out[0], idx, num, vbs, vbs, vs, vs_head, sm_scale * math.log2(math.e), H, n, n, S, S,
                       qs=qs, ks=ks, idx_ld=n, q_scale_ld=n, kv_scale_ld=n, wide=True)

    t_ref, t_ours, t_wide = _time(ref), _time(ours), _time(ours_wide)
    ref_out = ref()
    ours_wide()
    torch.cuda.synchronize()
    err = float((out.double() - ref_out.double()).norm() / ref_out.double().norm())
    print(f"\nrel-Frobenius(FP8 h3b wide-step vs BF16 reference) = {err:.4f}")
    assert err < 0.1
    _report(f"VSA forward config 4 (reference BF16 vs h3b E4M3, tile kernel), top-{k} of {n}", t_ref, t_ours,
            4.0 * S * (k * 64) * D * H, "TFLOP/s")
    _report(f"VSA forward config 4 (reference BF16 vs h3b E4M3, wide-step kernel), top-{k} of {n}", t_ref, t_wide,
            4.0 * S * (k * 64) * D * H, "TFLOP/s")
