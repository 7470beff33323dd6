"""Generates the golden fixtures of ``cases.py`` by running the REFERENCE's own kernels (``oracle/_ref/h3ref.so``,
built from the reference's ``h3fast.cu`` by ``oracle/ref_build/build_ref.py``) on a B200.

Run on a GPU box: ``python tests/golden/gen_golden.py``; it writes ``tests/golden/<case>.npz`` (and a copy under
``gpurun_out/golden/`` so a remote run can bring them back). Only the reference's outputs are stored.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from cases import CASES, outlier_matrix, rnq_inputs  # noqa: E402

from oracle.ref_build.build_ref import load  # noqa: E402


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).cpu().numpy()


def run_rnq(mod, cdll, C, rows, seed, branch, norm, fp4):
    d = {k: v.cuda() for k, v in rnq_inputs(C, rows, seed).items()}
    xo = torch.empty_like(d["x"])
    pad = (rows + 127) // 128 * 128
    h = torch.zeros(rows, C // 2 if fp4 else C, device="cuda", dtype=torch.uint8)
    hsf = torch.zeros(pad, C // 16, device="cuda", dtype=torch.uint8) if fp4 else None
    hs = torch.zeros(rows, device="cuda")
    y, sy, gate = (d["y"], d["sy"], d["gate"]) if branch else (None, None, None)
    nw, shift, scale = (d["nw"], d["shift"], d["scale"]) if norm else (None, None, None)
    hh = (h if fp4 else h.view(torch.float8_e4m3fn)) if norm else None
    if C == 5376:
        mod.resid_norm_quant(d["x"], y, sy, gate, d["idx"], nw, shift, scale, xo, hh, hsf, hs if norm else None,
                             1e-5)
    else:
        P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        rc = cdll.h3ref_resid_norm_quant_5120(
            P(d["x"]), P(y), P(sy), P(gate), gate.stride(0) if gate is not None else 0, P(d["idx"]), P(nw),
            P(shift), P(scale), scale.stride(0) if scale is not None else 0, P(xo), P(hh), P(hsf),
            P(hs) if norm else None, 1e-5, rows, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, rc
    torch.cuda.synchronize()
    out = {}
    if branch:
        out["xo"] = xo.view(torch.int16).cpu().numpy().view(np.uint16)
    if norm:
        out["h"] = _u8(h)
        out["hs"] = hs.cpu().numpy()
        if fp4:
            out["hsf"] = _u8(hsf)
    return out


def run_nvfp4(cdll, rows, K, seed, frac, mult, std):
    x = outlier_matrix(rows, K, seed, frac, mult, std).cuda()
    pad = (rows + 127) // 128 * 128
    q = torch.zeros(rows, K // 2, device="cuda", dtype=torch.uint8)
    sf = torch.zeros(pad, K // 16, device="cuda", dtype=torch.uint8)
    s = torch.zeros(1, device="cuda")
    ws = torch.zeros(64, device="cuda")
    rc = cdll.h3ref_quant_nvfp4_tensor(x.data_ptr(), rows, K, ws.data_ptr(), q.data_ptr(), sf.data_ptr(),
                                       s.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return {"q": _u8(q), "sf": _u8(sf), "s": s.cpu().numpy()}


def main() -> None:
    mod, cdll = load()
    if mod is None:
        raise SystemExit("oracle/_ref/h3ref.so is missing: run oracle/ref_build/build_ref.py where the reference is")
    outdirs = [HERE, ROOT / "gpurun_out" / "golden"]
    for dd in outdirs:
        dd.mkdir(parents=True, exist_ok=True)
    for name, (kind, p) in CASES.items():
        out = run_rnq(mod, cdll, **p) if kind == "rnq" else run_nvfp4(cdll, **p)
        for dd in outdirs:
            np.savez_compressed(dd / f"{name}.npz", **out)
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
