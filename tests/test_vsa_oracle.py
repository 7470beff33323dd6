"""CPU pins of the VSA oracle against the golden outputs of the reference's own kernels (top-k, prologue, gate)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from cases import GATE_CASES, PROLOGUE_CASES, TOPK_CASES, gate_inputs, prologue_inputs, topk_inputs
from oracle import quant as oq
from oracle import vsa as ov
from test_oracle import _golden, assert_codes


@pytest.mark.parametrize("name", list(TOPK_CASES))
def test_topk_oracle_matches_reference(name):
    p = TOPK_CASES[name]
    gold = _golden(name)
    sc = topk_inputs(p["heads"], p["n"], p["seed"], p["quantize"] or 1e6).numpy()
    idx, num = ov.topk_rows(sc, p["n"], p["n"], p["prefix"], p["spans"], p["split"])
    np.testing.assert_array_equal(num, gold["num"][0])
    for h in range(p["heads"]):
        for q in range(p["n"]):
            c = num[h, q]
            np.testing.assert_array_equal(idx[h, q, :c], gold["idx"][0, h, q, :c])


def test_topk_ties_go_to_lowest_column_and_negative_zero_sorts_low():
    sc = np.zeros((1, 8), dtype=np.float32)
    sc[0, [1, 5, 6]] = 1.0
    sc[0, 3] = -0.0
    idx, num = ov.topk_rows(sc.reshape(1, 8).repeat(8, 0), 8, 8, 0, [(0, 8, 4)], False)
    # three 1.0s, then the lowest-column +0.0 (column 0); -0.0 at column 3 ranks below +0.0
    np.testing.assert_array_equal(idx[0, 0, :4], [0, 1, 5, 6])


@pytest.mark.parametrize("name", list(PROLOGUE_CASES))
def test_prologue_oracle_matches_reference(name):
    p = PROLOGUE_CASES[name]
    gold = _golden(name)
    d = prologue_inputs(p["heads"], p["n_tiles"], p["seed"])
    bound = math.sqrt(128) / 448.0
    s_q = bound * d["wq"].float().abs().max().item()
    s_k = bound * d["wk"].float().abs().max().item()
    f = lambda t: t.float().numpy()  # noqa: E731
    ref = ov.qkv_prologue8(f(d["q"]), f(d["k"]), f(d["v"]), d["s1"].numpy(), d["tile_row0"].numpy(), d["vbs"].numpy(),
                           f(d["wq"]), f(d["wk"]), f(d["cos"]), f(d["sin"]), p["heads"], s_q, s_k)
    for key in ("qb", "kb", "vb"):
        got = oq.e4m3_decode(gold[key][0])
        want = oq.e4m3_decode(ref[key])
        close = np.abs(got - want) <= np.maximum(np.abs(want), 2 ** -6) * 0.126
        assert close.mean() > 0.999, (key, close.mean())
    np.testing.assert_allclose(gold["vs_blk"], ref["vs_blk"], rtol=1e-2)
    # tile means of the bf16-rounded values, same order as the kernel
    for t in range(p["n_tiles"]):
        r0, n = int(d["tile_row0"][t]), int(d["vbs"][t])
        for h in range(p["heads"]):
            np.testing.assert_allclose(gold["vp"][h, t], ov.tile_means(ref["v"][r0:r0 + n, h]), rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("name", list(GATE_CASES))
def test_gate_oracle_matches_reference(name):
    p = GATE_CASES[name]
    gold = _golden(name)
    d = gate_inputs(p["heads"], p["vbs"], p["seed"])
    f = lambda t: t.float().numpy()  # noqa: E731
    rows = int(sum(p["vbs"]))
    ref = ov.attn_gate_quant(f(d["ob"])[0], d["slot"].numpy(), rows, f(d["g"]), d["sg"].numpy(), f(d["oc"]),
                             fp4=p["fp4"])
    np.testing.assert_allclose(gold["sa"], ref["s"], rtol=4e-7)
    if p["fp4"]:
        assert_codes(oq.unpack_nibbles(gold["a"]), ref["codes"], ref["amb"], "gate nibbles")
        assert_codes(oq.unswizzle_sf(gold["asf"], rows, p["heads"] * 8), ref["sf_bits"], ref["sf_amb"], "gate sf")
    else:
        assert_codes(gold["a"], ref["codes"], ref["amb"], "gate fp8")
