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


def _round_f32_exact(x) -> np.float32:
    """Round an exact rational to float32, ties to even, by comparing the two float32 neighbours exactly."""
    from fractions import Fraction
    t = np.float32(float(x))  # within one float32 ulp of x
    best = None
    for cand in (np.nextafter(t, np.float32(-np.inf)), t, np.nextafter(t, np.float32(np.inf))):
        err = abs(Fraction(float(cand)) - x)
        even = (int(np.asarray(cand).view(np.uint32)) & 1) == 0
        if best is None or err < best[0] or (err == best[0] and even):
            best = (err, cand)
    return np.float32(best[1])


def test_fma32_is_correctly_rounded():
    """The oracle's float32 fused multiply-add (the tile scores' accumulation step) against exact rational
    arithmetic: random operands over a wide exponent range, plus constructed cases where the float64 sum lands exactly
    on a float32 midpoint and only the rounding error decides the direction."""
    from fractions import Fraction
    rng = np.random.default_rng(7)
    n = 4000
    a = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32)
    b = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32)
    c = (rng.standard_normal(n) * np.exp2(rng.integers(-40, 40, n))).astype(np.float32)
    # midpoint cases: a*b = +-half_ulp * (1 - 2^-36) exactly, so c + a*b lies 2^-36 half-ulps inside a float32
    # midpoint: float64 rounds the sum onto the midpoint itself and only the TwoSum error gives the direction
    m = 600
    base = rng.standard_normal(m).astype(np.float32)
    half_ulp = np.abs(np.spacing(base).astype(np.float64)) / 2
    a2 = np.full(m, 1.0 + 2.0 ** -18, dtype=np.float32)
    b2 = (half_ulp * (1.0 - 2.0 ** -18) * rng.choice([-1.0, 1.0], m)).astype(np.float32)
    c2 = base
    a = np.concatenate([a, a2])
    b = np.concatenate([b, b2])
    c = np.concatenate([c, c2])
    got = ov.fma32(a, b, c)
    for i in range(a.size):
        x = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        want = _round_f32_exact(x)
        assert got[i].view(np.uint32) == want.view(np.uint32), (i, a[i], b[i], c[i], got[i], want)


def test_tile_scores_fixed_order():
    """tile scores = one fused multiply-add per dimension, d ascending, then the scale: a direct scalar loop."""
    rng = np.random.default_rng(3)
    qp = rng.standard_normal((2, 5, 128)).astype(np.float32) * np.float32(0.1)
    kp = rng.standard_normal((2, 7, 128)).astype(np.float32) * np.float32(0.1)
    scale = 1.0 / math.sqrt(128)
    got = ov.tile_scores(qp, kp, scale)
    for h, i, j in [(0, 0, 0), (1, 4, 6), (0, 3, 2)]:
        acc = np.float32(0)
        for d in range(128):
            acc = ov.fma32(qp[h, i, d], kp[h, j, d], acc)
        assert got[h, i, j].view(np.uint32) == np.float32(acc * np.float32(scale)).view(np.uint32)


def test_topk_pairs_union_by_hand():
    """Two query tiles' selections merged: ascending union, membership bits, a pad tile selecting nothing."""
    n, n_ext = 5, 6
    sc = np.zeros((1, n, n), dtype=np.float32)
    sc[0, 0] = [5, 4, 3, 2, 1]   # tile 0 keeps 0, 1
    sc[0, 1] = [1, 2, 3, 4, 5]   # tile 1 keeps 3, 4
    sc[0, 2] = [1, 9, 1, 9, 1]   # tile 2 keeps 1, 3
    sc[0, 3] = [9, 1, 1, 1, 9]   # tile 3 keeps 0, 4
    sc[0, 4] = [2, 2, 2, 2, 2]   # tile 4 keeps 0, 1 (ties to the lowest column); tile 5 is padding
    u_idx, u_mem, u_num = ov.topk_pairs(sc, n, n_ext, 0, [(0, n, 2)])
    assert u_num.tolist() == [4, 4, 2]
    assert u_idx[0, :4].tolist() == [0, 1, 3, 4] and u_mem[0, :4].tolist() == [1, 1, 2, 2]
    assert u_idx[1, :4].tolist() == [0, 1, 3, 4] and u_mem[1, :4].tolist() == [2, 1, 1, 2]
    assert u_idx[2, :2].tolist() == [0, 1] and u_mem[2, :2].tolist() == [1, 1]
