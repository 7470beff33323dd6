"""GPU parity of the quantizers and weight packing.

Three references, strongest first:
  1. the golden outputs of the reference's own kernels (tests/golden, bit-exact);
  2. the reference kernels themselves, live, from oracle/_ref when that prebuilt file is present (bit-exact on large
     random inputs);
  3. the CPU oracle (bit-exact outside its documented ambiguity window; the only reference for the LayerNorm variant
     and for the plain per-token quantizer, which the reference does not have).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from cases import CASES, outlier_matrix, rnq_inputs
from oracle import quant as oq
from test_oracle import _golden, assert_codes, assert_scales

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _u8(t):
    return t.contiguous().view(torch.uint8).cpu().numpy()


def run_rnq(ops, d, C, rows, branch, norm, fp4, norm_kind="rms"):
    d = {k: v.to(DEV) for k, v in d.items()}
    xo = torch.empty_like(d["x"])
    h = torch.zeros(rows, C // 2 if fp4 else C, device=DEV, dtype=torch.uint8)
    hsf = torch.zeros(ops.sf_rows(rows), C // 16, device=DEV, dtype=torch.uint8) if fp4 else None
    hs = torch.zeros(rows, device=DEV)
    y, sy, gate = (d["y"], d["sy"], d["gate"]) if branch else (None, None, None)
    nw = d["nw"] if (norm and norm_kind == "rms") else None
    shift, scale = (d["shift"], d["scale"]) if norm else (None, None)
    ops.resid_norm_quant(d["x"], y, sy, gate, d["idx"], nw, shift, scale, xo, h if norm else None, hsf,
                         hs if norm else None, 1e-5, norm=norm_kind if norm else "none")
    torch.cuda.synchronize()
    return xo, h, hsf, hs


@pytest.mark.parametrize("name", [n for n, (k, _) in CASES.items() if k == "rnq"])
def test_row_quantizer_bit_exact_vs_reference_golden(ops, name):
    p = CASES[name][1]
    gold = _golden(name)
    d = rnq_inputs(p["C"], p["rows"], p["seed"])
    xo, h, hsf, hs = run_rnq(ops, d, p["C"], p["rows"], p["branch"], p["norm"], p["fp4"])
    if p["branch"]:
        np.testing.assert_array_equal(xo.view(torch.int16).cpu().numpy().view(np.uint16), gold["xo"])
    if p["norm"]:
        np.testing.assert_array_equal(_u8(h), gold["h"])
        np.testing.assert_array_equal(hs.cpu().numpy().view(np.uint32), gold["hs"].view(np.uint32))
        if p["fp4"]:
            np.testing.assert_array_equal(_u8(hsf), gold["hsf"])


@pytest.mark.parametrize("name", [n for n, (k, _) in CASES.items() if k == "nvfp4"])
def test_tensor_nvfp4_bit_exact_vs_reference_golden(ops, name):
    p = CASES[name][1]
    gold = _golden(name)
    rows, K = p["rows"], p["K"]
    x = outlier_matrix(rows, K, p["seed"], p["frac"], p["mult"], p["std"]).to(DEV)
    q = torch.empty(rows, K // 2, device=DEV, dtype=torch.uint8)
    sf = torch.full((ops.sf_rows(rows), K // 16), 0xAB, device=DEV, dtype=torch.uint8)  # padding must be rewritten
    s = torch.empty(1, device=DEV)
    ws = torch.empty(ops.workspace_bytes(), device=DEV, dtype=torch.uint8)
    ops.quant_nvfp4(x, q, sf, s, ws)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_u8(q), gold["q"])
    np.testing.assert_array_equal(_u8(sf), gold["sf"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), gold["s"].view(np.uint32))


@pytest.mark.parametrize("rows,K", [(37, 320), (130, 3072), (129, 13824)])
def test_tensor_nvfp4_widths_vs_oracle(ops, rows, K):
    """Per-tensor NVFP4 at widths that are not multiples of the quantizer's 256-element warp unit (K = 320: a
    64-element tail unit), BASELINE's 3072 and the FFN width 13824, and row counts that leave scale padding rows."""
    x = outlier_matrix(rows, K, 300 + K, 0.005, 30.0)
    xd = x.to(DEV)
    q = torch.empty(rows, K // 2, device=DEV, dtype=torch.uint8)
    sf = torch.full((ops.sf_rows(rows), K // 16), 0xAB, device=DEV, dtype=torch.uint8)  # padding must be rewritten
    s = torch.empty(1, device=DEV)
    ops.quant_nvfp4(xd, q, sf, s, torch.empty(ops.workspace_bytes(), device=DEV, dtype=torch.uint8))
    torch.cuda.synchronize()
    rq, rsf, rs, amb, sf_amb = oq.quant_nvfp4_tensor(x.float().numpy())
    np.testing.assert_allclose(s.cpu().numpy(), np.float32(rs).reshape(1), rtol=4e-7)  # fast-math division
    assert_codes(oq.unpack_nibbles(_u8(q)), oq.unpack_nibbles(rq), amb, "tensor nvfp4 nibbles")
    got_bits = oq.unswizzle_sf(_u8(sf), rows, K // 16)
    want_bits = oq.unswizzle_sf(rsf, rows, K // 16)
    assert_codes(got_bits, want_bits, sf_amb, "tensor nvfp4 scales")
    pad = _u8(sf).reshape(-1)[oq.sf_atom_offset(np.arange(rows, ops.sf_rows(rows))[:, None],
                                                 np.arange(K // 16)[None, :], K // 16).reshape(-1)]
    assert (pad == 0).all()


def _ref():
    from oracle.ref_build.build_ref import load
    mod, cdll = load()
    if mod is None:
        pytest.skip("oracle/_ref/h3ref.so not present (built only where the reference sources are)")
    return mod, cdll


@pytest.mark.parametrize("C,branch,fp4", [(5376, True, False), (5376, True, True), (5120, True, False),
                                          (5120, False, True), (5120, True, True)])
def test_row_quantizer_bit_exact_vs_live_reference_large(ops, C, branch, fp4):
    mod, cdll = _ref()
    rows = 3001  # not a multiple of 128: the NVFP4 scale buffer has padding rows
    d = rnq_inputs(C, rows, seed=100 + C + 2 * fp4 + branch)
    xo, h, hsf, hs = run_rnq(ops, d, C, rows, branch, True, fp4)
    dd = {k: v.to(DEV) for k, v in d.items()}
    rxo = torch.empty_like(dd["x"])
    rh = torch.zeros_like(h)
    rhsf = torch.zeros_like(hsf) if fp4 else None
    rhs = torch.zeros_like(hs)
    y, sy, gate = (dd["y"], dd["sy"], dd["gate"]) if branch else (None, None, None)
    if C == 5376:
        mod.resid_norm_quant(dd["x"], y, sy, gate, dd["idx"], dd["nw"], dd["shift"], dd["scale"], rxo,
                             rh if fp4 else rh.view(torch.float8_e4m3fn), rhsf, rhs, 1e-5)
    else:
        P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        assert cdll.h3ref_resid_norm_quant_5120(P(dd["x"]), P(y), P(sy), P(gate), dd["gate"].stride(0), P(dd["idx"]),
                                                P(dd["nw"]), P(dd["shift"]), P(dd["scale"]), dd["scale"].stride(0),
                                                P(rxo), P(rh), P(rhsf), P(rhs), 1e-5, rows,
                                                torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    if branch:
        assert torch.equal(xo.view(torch.int16), rxo.view(torch.int16))
    assert torch.equal(h, rh)
    assert torch.equal(hs.view(torch.int32), rhs.view(torch.int32))
    if fp4:
        assert torch.equal(hsf, rhsf)


def test_tensor_nvfp4_bit_exact_vs_live_reference_large(ops):
    _, cdll = _ref()
    rows, K = 4099, 5120
    x = outlier_matrix(rows, K, 77, 0.005, 30.0).to(DEV)
    q = torch.empty(rows, K // 2, device=DEV, dtype=torch.uint8)
    sf = torch.zeros(ops.sf_rows(rows), K // 16, device=DEV, dtype=torch.uint8)
    s = torch.empty(1, device=DEV)
    ops.quant_nvfp4(x, q, sf, s, torch.empty(256, device=DEV, dtype=torch.uint8))
    rq, rsf, rs = torch.zeros_like(q), torch.zeros_like(sf), torch.zeros_like(s)
    ws = torch.zeros(64, device=DEV)
    assert cdll.h3ref_quant_nvfp4_tensor(x.data_ptr(), rows, K, ws.data_ptr(), rq.data_ptr(), rsf.data_ptr(),
                                         rs.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(sf, rsf) and torch.equal(s, rs)


def test_layernorm_variant_vs_oracle(ops):
    C, rows = 5120, 257
    d = rnq_inputs(C, rows, seed=11)
    for fp4 in (False, True):
        xo, h, hsf, hs = run_rnq(ops, d, C, rows, True, True, fp4, norm_kind="layer")
        f = lambda t: t.float().numpy()  # noqa: E731
        out = oq.resid_norm_quant(f(d["x"]), f(d["y"]), d["sy"].numpy(), f(d["gate"]), d["idx"].numpy(), None,
                                  f(d["shift"]), f(d["scale"]), 1e-5, norm="layer", fp4=fp4)
        np.testing.assert_array_equal(xo.float().cpu().numpy(), out["xo"])
        assert_scales(hs.cpu().numpy(), out["hs"], "layernorm row scales", rtol=2e-6)
        if fp4:
            assert_codes(oq.unswizzle_sf(_u8(hsf), rows, C // 16), out["sf_bits"], out["sf_amb"], "ln sf")
            assert_codes(oq.unpack_nibbles(_u8(h)), out["codes"], out["amb"], "ln nibbles")
        else:
            assert_codes(_u8(h), out["h"], out["amb"], "ln fp8")


@pytest.mark.parametrize("C", [3072, 4096, 5120, 5376])
def test_layernorm_shared_table_every_width(ops, C):
    """The runner's LayerNorm form: one adaLN table row for all tokens (idx NULL, the table kept in shared memory), at
    every supported width (the CTA's row-buffer count depends on C), FP8 and NVFP4, against the oracle."""
    rows = 131
    d = rnq_inputs(C, rows, seed=40 + C % 97)
    f = lambda t: t.float().numpy()  # noqa: E731
    shift, scale = d["shift"][0:1].contiguous(), d["scale"][0:1].contiguous()
    for fp4 in (False, True):
        x = d["x"].to(DEV)
        xo = torch.empty_like(x)
        h = torch.zeros(rows, C // 2 if fp4 else C, device=DEV, dtype=torch.uint8)
        hsf = torch.zeros(ops.sf_rows(rows), C // 16, device=DEV, dtype=torch.uint8) if fp4 else None
        hs = torch.zeros(rows, device=DEV)
        ops.resid_norm_quant(x, None, None, None, None, None, shift.to(DEV), scale.to(DEV), xo, h, hsf, hs, 1e-6,
                             norm="layer")
        torch.cuda.synchronize()
        out = oq.resid_norm_quant(f(d["x"]), None, None, None, np.zeros(rows, dtype=np.int32), None, f(shift),
                                  f(scale), 1e-6, norm="layer", fp4=fp4)
        assert_scales(hs.cpu().numpy(), out["hs"], f"layernorm row scales C={C}", rtol=2e-6)
        if fp4:
            assert_codes(oq.unswizzle_sf(_u8(hsf), rows, C // 16), out["sf_bits"], out["sf_amb"], f"ln sf C={C}")
            assert_codes(oq.unpack_nibbles(_u8(h)), out["codes"], out["amb"], f"ln nibbles C={C}")
        else:
            assert_codes(_u8(h), out["h"], out["amb"], f"ln fp8 C={C}")


@pytest.mark.parametrize("C,rows,per_token", [(5120, 4999, False), (5376, 3001, True), (3072, 2311, True)])
def test_layernorm_row_ring_wraps(ops, C, rows, per_token):
    """Row counts above (resident CTAs x ring stages), so every CTA refills and re-uses its row buffers several times
    (the mbarrier parity flips), with one shared table row or a per-token table row (idx), NVFP4 and FP8."""
    d = rnq_inputs(C, rows, seed=7 + C % 89)
    f = lambda t: t.float().numpy()  # noqa: E731
    if per_token:
        idx = d["idx"]
        shift, scale = d["shift"].contiguous(), d["scale"].contiguous()
    else:
        idx = None
        shift, scale = d["shift"][0:1].contiguous(), d["scale"][0:1].contiguous()
    oidx = np.zeros(rows, dtype=np.int32) if idx is None else idx.numpy()
    for fp4 in (True, False):
        x = d["x"].to(DEV)
        h = torch.zeros(rows, C // 2 if fp4 else C, device=DEV, dtype=torch.uint8)
        hsf = torch.zeros(ops.sf_rows(rows), C // 16, device=DEV, dtype=torch.uint8) if fp4 else None
        hs = torch.zeros(rows, device=DEV)
        ops.resid_norm_quant(x, None, None, None, None if idx is None else idx.to(DEV), None, shift.to(DEV),
                             scale.to(DEV), x, h, hsf, hs, 1e-6, norm="layer")
        ops.check_status()
        out = oq.resid_norm_quant(f(d["x"]), None, None, None, oidx, None, f(shift), f(scale), 1e-6, norm="layer",
                                  fp4=fp4)
        assert_scales(hs.cpu().numpy(), out["hs"], f"ring row scales C={C}", rtol=2e-6)
        if fp4:
            assert_codes(oq.unswizzle_sf(_u8(hsf), rows, C // 16), out["sf_bits"], out["sf_amb"], f"ring sf C={C}")
            assert_codes(oq.unpack_nibbles(_u8(h)), out["codes"], out["amb"], f"ring nibbles C={C}")
        else:
            assert_codes(_u8(h), out["h"], out["amb"], f"ring fp8 C={C}")


def test_fp8_rows_vs_oracle_config1(ops):
    # BASELINE config 1 activations: [2048 x 3072] N(0,1) with 1% of columns x20
    x = outlier_matrix(2048, 3072, 0, 0.01, 20.0)
    q = torch.empty(2048, 3072, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(2048, device=DEV)
    ops.quant_fp8_rows(x.to(DEV), q, s)
    torch.cuda.synchronize()
    codes, s_ref, amb = oq.quant_fp8_rows(x.float().numpy())
    assert_scales(s.cpu().numpy(), s_ref, "fp8 row scales", rtol=2e-7)
    assert_codes(_u8(q), codes, amb, "fp8 row codes")


def test_fp8_rows_edge_cases(ops):
    x = torch.zeros(3, 256, dtype=torch.bfloat16)
    x[1, 7] = 1e-30  # below bf16 normal range: rounds to a tiny value
    x[2] = 1000.0
    q = torch.empty(3, 256, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(3, device=DEV)
    ops.quant_fp8_rows(x.to(DEV), q, s)
    torch.cuda.synchronize()
    assert s[0].item() == pytest.approx(1 / (448 * 512))  # all-zero row takes the floor scale
    assert (q[0].view(torch.uint8) == 0).all()
    assert q[2].float().eq(448).all()
    # empty input is a no-op
    ops.quant_fp8_rows(torch.empty(0, 256, device=DEV, dtype=torch.bfloat16), q[:0], s[:0])


@pytest.mark.parametrize("gran", ["channel", "tensor"])
def test_fp8_weight_packing_bit_exact_vs_restatement(ops, gran):
    w = (torch.randn(3072, 3072, generator=torch.Generator().manual_seed(5)) * 0.02).bfloat16()
    w[17] = 0  # an all-zero output channel takes FP8_MIN_SCALE
    wq, ws = ops.quantize_fp8_weight(w.to(DEV), gran)
    rq, rs = oq.quantize_fp8_weight(w, gran)
    assert torch.equal(wq.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(ws.cpu(), rs)


def test_nvfp4_weight_packing(ops):
    N, K = 1000, 5120  # N not a multiple of 128
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(6)) * 0.02).bfloat16()
    wq, wsf, ws = ops.pack_nvfp4_weight(w.to(DEV))
    torch.cuda.synchronize()
    q, sf, s, amb, sf_amb = oq.quant_nvfp4_tensor(w.float().numpy())
    assert_scales(ws.cpu().numpy(), np.array([s]), "weight tensor scale")
    assert_codes(oq.unswizzle_sf(_u8(wsf), N, K // 16), oq.unswizzle_sf(sf, N, K // 16), sf_amb, "weight sf")
    assert_codes(oq.unpack_nibbles(_u8(wq)), oq.unpack_nibbles(q), amb, "weight nibbles")


@pytest.mark.parametrize("case", ["fp8pack_small", "fp8pack_3072"])
@pytest.mark.parametrize("gran", ["channel", "tensor"])
def test_fp8_weight_packing_vs_reference_run(ops, case, gran):
    """h3b_pack_weight_fp8 against the reference's own quantize_fp8_weight (patch:384-394) run on the same seeded
    weights (golden fixture from tests/golden/gen_fp8_pack_golden.py): codes and scales bit for bit."""
    from cases import FP8_PACK_CASES, fp8_pack_weight
    gold = np.load(Path(__file__).resolve().parent / "golden" / "fp8_weight_pack.npz")
    w = fp8_pack_weight(**FP8_PACK_CASES[case]).to(DEV)
    q, s = ops.quantize_fp8_weight(w, gran)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), gold[f"{case}.{gran}.q"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), gold[f"{case}.{gran}.s"].view(np.uint32))
