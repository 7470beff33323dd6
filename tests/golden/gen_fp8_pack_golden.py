"""Generates ``tests/golden/fp8_weight_pack.npz`` from the REFERENCE's own ``quantize_fp8_weight``.

The function is added to FastVideo's ``fastvideo/layers/quantization/fp8_config.py`` by the reference's patch
(patches/fastvideo-a01c50a.patch:384-394); FastVideo itself is not installed here. This script reads the patch text,
takes the added lines of that function unchanged, and runs them with torch on the CPU. The three module constants it
uses come from FastVideo's fp8_config module, which the reference does not vendor: ``FP8_DTYPE`` is
``torch.float8_e4m3fn``, ``FP8_MAX`` its largest finite value (448), and ``FP8_MIN_SCALE`` the floor this library
uses for an all-zero channel, 1 / (448 * 512) (the reference kernels' ``kMinScale``, h3fast.cu:23). Inputs are the
seeded weights of ``cases.FP8_PACK_CASES``; the fixture holds the reference's codes and scales. Run in a checkout
that has the reference source tree: ``python tests/golden/gen_fp8_pack_golden.py [REFERENCE_DIR]``.
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

from cases import FP8_PACK_CASES, fp8_pack_weight  # noqa: E402

from oracle.ref_build.build_ref import reference_root  # noqa: E402


def reference_quantize_fp8_weight(root: str | None = None):
    ref = reference_root(root)
    if ref is None:
        raise SystemExit("the reference source tree was not found (argument, $H3_REFERENCE or ../reference)")
    patch = (ref / "patches" / "fastvideo-a01c50a.patch").read_text().splitlines()
    start = next(i for i, ln in enumerate(patch) if ln.startswith("+def quantize_fp8_weight("))
    body = []
    for ln in patch[start:]:
        if body and ln.startswith("+def ") or (body and not ln.startswith("+")):
            break
        body.append(ln[1:])
    ns = {"torch": torch, "FP8_DTYPE": torch.float8_e4m3fn, "FP8_MAX": float(torch.finfo(torch.float8_e4m3fn).max),
          "FP8_MIN_SCALE": 1.0 / (448.0 * 512.0)}
    exec(compile("from __future__ import annotations\n" + "\n".join(body), "quantize_fp8_weight", "exec"), ns)
    return ns["quantize_fp8_weight"]


def main() -> None:
    fn = reference_quantize_fp8_weight(sys.argv[1] if len(sys.argv) > 1 else None)
    out = {}
    for name, c in FP8_PACK_CASES.items():
        w = fp8_pack_weight(**c)
        for gran in ("channel", "tensor"):
            q, s = fn(w, gran)
            out[f"{name}.{gran}.q"] = q.view(torch.uint8).numpy()
            out[f"{name}.{gran}.s"] = s.float().numpy()
    np.savez_compressed(HERE / "fp8_weight_pack.npz", **out)
    print("wrote", HERE / "fp8_weight_pack.npz", sorted(out))


if __name__ == "__main__":
    main()
