"""Generates ``tests/golden/lora_on_grid.npz`` from the REFERENCE's own LoRA helpers.

``_on_grid`` and ``_adapter``'s scale rule live in fastvideo/models/dits/h3fast/__init__.py (:63-92) as pure torch,
but that module imports FastVideo, which is not installed here. This script therefore parses the reference file,
takes the module constants ``_FP8``/``_FP8_MAX`` and the function ``_on_grid`` from its syntax tree unchanged, and runs
them with torch on the CPU on the seeded inputs of ``cases.LORA_CASES`` (the merge ``W.float() + scale * B @ A`` done
with ``addmm_`` as ``_merged_fp8`` does, :354-376). Only the inputs the tests need and the reference's outputs are
stored. Run in a checkout that has the reference source tree: ``python tests/golden/gen_lora_golden.py``
($H3_REFERENCE names the tree when it is not in the default place of ``oracle.ref_build.build_ref``).
"""
from __future__ import annotations

import ast
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from cases import LORA_CASES, lora_inputs  # noqa: E402

from oracle.ref_build.build_ref import reference_root  # noqa: E402


def reference_helpers() -> dict:
    src = reference_root() / "fastvideo" / "models" / "dits" / "h3fast" / "__init__.py"
    tree = ast.parse(src.read_text())
    keep = []
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) in ("_FP8", "_FP8_MAX") for t in node.targets):
            keep.append(node)
        if isinstance(node, ast.FunctionDef) and node.name == "_on_grid":
            keep.append(node)
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(src), "exec"), ns)
    return ns


def main() -> None:
    ns = reference_helpers()
    out = {}
    for name, c in LORA_CASES.items():
        d = lora_inputs(c["N"], c["K"], c["rank"], c["seed"], c["per_row"], c["big_every"], c["big"])
        rank, alpha, strength = c["rank"], c["alpha"], c["strength"]
        scale = strength * (float(alpha) / float(rank) if alpha != rank else 1.0)
        merged = d["w"].float()
        merged.addmm_(d["B"].float(), d["A"].float(), alpha=scale)
        q, s = ns["_on_grid"](merged, d["base_scale"])
        out[f"{name}.merged"] = merged.numpy()
        out[f"{name}.base_scale"] = d["base_scale"].numpy()
        out[f"{name}.lora_scale"] = np.float64(scale)
        out[f"{name}.q"] = q.view(torch.uint8).numpy()
        out[f"{name}.s"] = s.float().numpy()
    np.savez_compressed(HERE / "lora_on_grid.npz", **out)
    print("wrote", HERE / "lora_on_grid.npz", sorted(out))


if __name__ == "__main__":
    main()
