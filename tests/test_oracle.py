"""CPU tests of the oracle: encoder round trips, the scale-factor layout, the reduction-tree emulation, and the pin of
the oracle against the golden outputs of the reference's own kernels (tests/golden/*.npz)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import CASES, outlier_matrix, rnq_inputs
from conftest import ROOT
from oracle import quant as oq

GOLDEN = ROOT / "tests" / "golden"


def test_e4m3_encoder_matches_torch_and_saturates():
    x = np.array([0, 1e-9, 0.0019, 1.0, 1.0625, 447.9, 448, 460, 1e6, -3.3, -1e6], dtype=np.float32)
    codes = oq.e4m3_encode(x)
    back = oq.e4m3_decode(codes)
    assert back[-1] == -448 and back[-4] == 448 and back[-3] == 448  # saturating, not NaN
    np.testing.assert_array_equal(codes[:7], torch.from_numpy(x[:7]).to(torch.float8_e4m3fn).view(torch.uint8).numpy())


def test_e2m1_encoder_ties_to_even_and_saturates():
    x = np.array([0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.01, 100, -0.1, -6], dtype=np.float32)
    got = oq.e2m1_decode(oq.e2m1_encode(x))
    np.testing.assert_array_equal(got, [0, 0.5, 1, 1, 2, 2, 4, 4, 6, 6, -0.0, -6])
    assert oq.e2m1_encode(np.float32(-0.1)) == 8  # sign kept on a negative value that rounds to zero


def test_e2m1_round_trip_all_codes():
    codes = np.arange(16, dtype=np.uint8)
    np.testing.assert_array_equal(oq.e2m1_encode(oq.e2m1_decode(codes)), codes)


def test_sf_layout_is_a_bijection_onto_the_padded_buffer():
    rows, cols = 300, 20
    r, c = np.meshgrid(np.arange(384), np.arange(cols), indexing="ij")
    off = oq.sf_atom_offset(r, c, cols)
    assert sorted(off.ravel().tolist()) == list(range(384 * cols))
    bits = np.random.default_rng(0).integers(0, 256, (rows, cols), dtype=np.uint8)
    np.testing.assert_array_equal(oq.unswizzle_sf(oq.swizzle_sf(bits), rows, cols), bits)


def test_sf_layout_matches_the_reference_test_formula():
    # tests/test_kernels.py:94 (reference): (r//128)*(K//64)*512 + (c//4)*512 + (r%32)*16 + ((r%128)//32)*4 + c%4
    r, c = np.meshgrid(np.arange(256), np.arange(8), indexing="ij")
    K = 128
    ref = (r // 128) * (K // 64) * 512 + (c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)
    np.testing.assert_array_equal(oq.sf_atom_offset(r, c, K // 16), ref)


def test_butterfly_tree_matches_an_explicit_shuffle_emulation():
    rng = np.random.default_rng(1)
    lanes = rng.standard_normal(32).astype(np.float32) * np.float32(1e3)
    v = lanes.copy()
    for o in (16, 8, 4, 2, 1):
        v = np.array([np.float32(v[l] + v[l ^ o]) for l in range(32)], dtype=np.float32)
    assert len(set(v.tolist())) == 1
    assert oq.butterfly_sum(lanes[None])[0] == v[0]


def test_quantize_fp8_weight_restatement_rounds_scale_to_weight_dtype():
    w = (torch.randn(8, 64, generator=torch.Generator().manual_seed(0)) * 0.02).bfloat16()
    q, s = oq.quantize_fp8_weight(w, "channel")
    assert q.dtype == torch.float8_e4m3fn and s.shape == (8,) and s.dtype == torch.float32
    sbf = s.to(torch.bfloat16).float()
    np.testing.assert_array_equal((w.float() / sbf[:, None]).bfloat16().clamp(-448, 448).to(torch.float8_e4m3fn)
                                  .view(torch.uint8).numpy(), q.view(torch.uint8).numpy())
    qt, st = oq.quantize_fp8_weight(w, "tensor")
    assert st.shape == (1,)


# ------------------------------------------------------------------------------------------------ golden pinning
def _golden(name):
    path = GOLDEN / f"{name}.npz"
    assert path.exists(), f"missing golden fixture {path} (generate with tests/golden/gen_golden.py on a B200)"
    return dict(np.load(path))


def _f(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def assert_codes(got: np.ndarray, want: np.ndarray, amb: np.ndarray, what: str, max_soft_frac: float = 5e-3,
                 max_amb_frac: float = 2e-2):
    """Equal everywhere outside the ambiguity mask; inside it (values within DELTA of a rounding boundary, where the
    reference's fast-math divisions may round either way -- with bf16 inputs many values sit exactly on a tie) only a
    small fraction may differ, and the mask itself must stay a small fraction of the codes."""
    assert got.shape == want.shape, (what, got.shape, want.shape)
    diff = got != want
    hard = diff & ~amb
    assert not hard.any(), f"{what}: {int(hard.sum())} of {got.size} codes differ outside the ambiguity window"
    assert amb.mean() <= max_amb_frac, f"{what}: ambiguity window covers {amb.mean():.2e} of the codes"
    assert diff.mean() <= max_soft_frac, f"{what}: {diff.mean():.2e} of the codes differ inside the window"


def assert_scales(got: np.ndarray, want: np.ndarray, what: str, rtol: float = 4e-7):
    np.testing.assert_allclose(got, want, rtol=rtol, atol=0, err_msg=what)


@pytest.mark.parametrize("name", [n for n, (k, _) in CASES.items() if k == "rnq"])
def test_oracle_matches_reference_row_kernel(name):
    p = CASES[name][1]
    gold = _golden(name)
    d = rnq_inputs(p["C"], p["rows"], p["seed"])
    kw = dict(x=_f(d["x"]), idx=d["idx"].numpy(), eps=1e-5, fp4=p["fp4"])
    if p["branch"]:
        kw.update(y=_f(d["y"]), sy=d["sy"].numpy(), gate=_f(d["gate"]))
    if p["norm"]:
        kw.update(nw=_f(d["nw"]), shift=_f(d["shift"]), scale=_f(d["scale"]), norm="rms")
    else:
        kw.update(norm="none")
    out = oq.resid_norm_quant(**kw)
    if p["branch"]:
        want_xo = oq.bf16_bits_to_f32(gold["xo"])
        np.testing.assert_array_equal(out["xo"], want_xo)
    if p["norm"]:
        assert_scales(out["hs"], gold["hs"], f"{name} row scales")
        if p["fp4"]:
            got_bits = out["sf_bits"]
            want_bits = oq.unswizzle_sf(gold["hsf"], p["rows"], p["C"] // 16)
            assert_codes(got_bits, want_bits, out["sf_amb"], f"{name} block scales")
            assert_codes(out["codes"], oq.unpack_nibbles(gold["h"]), out["amb"], f"{name} nibbles")
        else:
            assert_codes(out["h"], gold["h"], out["amb"], f"{name} fp8 codes")


@pytest.mark.parametrize("name", [n for n, (k, _) in CASES.items() if k == "nvfp4"])
def test_oracle_matches_reference_tensor_nvfp4(name):
    p = CASES[name][1]
    gold = _golden(name)
    x = outlier_matrix(p["rows"], p["K"], p["seed"], p["frac"], p["mult"], p["std"])
    q, sf, s, amb, sf_amb = oq.quant_nvfp4_tensor(_f(x))
    assert_scales(np.array([s]), gold["s"], f"{name} tensor scale")
    rows, K = p["rows"], p["K"]
    assert_codes(oq.unswizzle_sf(sf, rows, K // 16), oq.unswizzle_sf(gold["sf"], rows, K // 16), sf_amb,
                 f"{name} block scales")
    assert_codes(oq.unpack_nibbles(q), oq.unpack_nibbles(gold["q"]), amb, f"{name} nibbles")
    # padding rows of the scale buffer (interleaved inside the 128-row atoms) are zero in both
    pad = sf.shape[0]
    assert not oq.unswizzle_sf(sf, pad, K // 16)[rows:].any()
    assert not oq.unswizzle_sf(gold["sf"], pad, K // 16)[rows:].any()
