"""Generates the golden fixtures of ``cases.py`` by running the REFERENCE's own kernels (``oracle/_ref/h3ref.so``,
built from the reference's ``h3fast.cu`` by ``oracle/ref_build/build_ref.py``) on a B200.

Run on a GPU box: ``python tests/golden/gen_golden.py``; it writes ``tests/golden/<case>.npz`` (and a copy under
the repository's returned-output folder, so a remote run can bring them back). Only the reference's outputs are
stored.
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

from cases import (CASES, GATE_CASES, PROLOGUE_CASES, TOPK_CASES, gate_inputs, outlier_matrix,  # noqa: E402
                   prologue_inputs, rnq_inputs, topk_inputs)

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


def run_topk(mod, heads, n, seed, quantize, prefix, spans, split):
    sc = (topk_inputs(heads, n, seed, quantize) if quantize else topk_inputs(heads, n, seed, 1e6)).cuda()
    idx = torch.full((1, heads, n, n), -1, device="cuda", dtype=torch.int32)
    num = torch.zeros(1, heads, n, device="cuda", dtype=torch.int32)
    mod.topk_rows(sc, n, n, prefix, [a for a, _, _ in spans], [b for _, b, _ in spans], [c for _, _, c in spans], idx,
                  num, split)
    torch.cuda.synchronize()
    kmax = int(num.max().item())
    return {"idx": idx[..., :kmax].cpu().numpy(), "num": num.cpu().numpy()}


def prologue_static_scales(d):
    """The runner's static Q/K scales: sqrt(128) * max|w| / 448 (fastvideo/models/dits/h3fast/__init__.py:295-302)."""
    import math
    bound = math.sqrt(128) / 448.0
    return bound * d["wq"].float().abs().max().item(), bound * d["wk"].float().abs().max().item()


def run_prologue(mod, heads, n_tiles, seed):
    d = {k: v.cuda() for k, v in prologue_inputs(heads, n_tiles, seed).items()}
    n_ext = n_tiles + n_tiles % 2
    rows_pad = n_ext * 64
    s_q, s_k = prologue_static_scales(d)
    z = lambda *sh, dt=torch.uint8: torch.zeros(*sh, device="cuda", dtype=dt)  # noqa: E731
    qb, kb, vb = z(1, heads, rows_pad, 128), z(1, heads, rows_pad, 128), z(1, heads, rows_pad, 128)
    vs_blk = torch.ones(heads, n_ext, device="cuda")
    vs_head = torch.zeros(heads, device="cuda")
    qp, kp, vp = (z(heads, n_tiles, 128, dt=torch.float32) for _ in range(3))
    mod.qkv_prologue8(d["q"], d["k"], d["v"], d["s1"], d["tile_row0"], d["vbs"], d["wq"], d["wk"], d["cos"], d["sin"],
                      1.0 / s_q, 1.0 / s_k, qb, kb, vb, vs_blk, vs_head, qp, kp, vp, heads, n_tiles, 64, 1e-5,
                      None, None, None)
    torch.cuda.synchronize()
    return {"qb": qb.cpu().numpy(), "kb": kb.cpu().numpy(), "vb": vb.cpu().numpy(), "vs_blk": vs_blk.cpu().numpy(),
            "vs_head": vs_head.cpu().numpy(), "qp": qp.cpu().numpy(), "kp": kp.cpu().numpy(), "vp": vp.cpu().numpy()}


def run_gate(cdll, heads, vbs, seed, fp4):
    d = {k: v.cuda() for k, v in gate_inputs(heads, vbs, seed).items()}
    rows = int(sum(vbs))
    W = heads * 128
    a = torch.zeros(rows, W // 2 if fp4 else W, device="cuda", dtype=torch.uint8)
    asf = torch.zeros(128, W // 16, device="cuda", dtype=torch.uint8) if fp4 else None
    sa = torch.zeros(rows, device="cuda")
    rc = cdll.h3ref_attn_gate_quant_5120(d["ob"].data_ptr(), d["g"].data_ptr(), d["sg"].data_ptr(), d["oc"].data_ptr(),
                                         d["slot"].data_ptr(), d["ob"].shape[-2], len(vbs), 64, a.data_ptr(),
                                         asf.data_ptr() if fp4 else None, sa.data_ptr(), rows,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    out = {"a": a.cpu().numpy(), "sa": sa.cpu().numpy()}
    if fp4:
        out["asf"] = asf.cpu().numpy()
    return out


def main() -> None:
    mod, cdll = load()
    if mod is None:
        raise SystemExit("oracle/_ref/h3ref.so is missing: run oracle/ref_build/build_ref.py where the reference is")
    args = sys.argv[1:]
    extra = []
    if "--also-to" in args:  # a second copy of every fixture (e.g. a folder a remote run sends back)
        i = args.index("--also-to")
        extra = [Path(args[i + 1])]
        del args[i:i + 2]
    outdirs = [HERE, *extra]
    for dd in outdirs:
        dd.mkdir(parents=True, exist_ok=True)
    jobs = [(name, (lambda p=p, kind=kind: run_rnq(mod, cdll, **p) if kind == "rnq" else run_nvfp4(cdll, **p)))
            for name, (kind, p) in CASES.items()]
    jobs += [(name, (lambda p=p: run_topk(mod, **p))) for name, p in TOPK_CASES.items()]
    jobs += [(name, (lambda p=p: run_prologue(mod, **p))) for name, p in PROLOGUE_CASES.items()]
    jobs += [(name, (lambda p=p: run_gate(cdll, **p))) for name, p in GATE_CASES.items()]
    only = set(args)
    for name, job in jobs:
        if only and name not in only:
            continue
        out = job()
        for dd in outdirs:
            np.savez_compressed(dd / f"{name}.npz", **out)
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
