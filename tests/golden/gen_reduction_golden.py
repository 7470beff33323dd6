"""Generates ``tests/golden/reduction.npz`` from the REFERENCE's own token-reduction functions.

fastvideo/models/dits/minimax_h3_token_reduction.py imports FastVideo (not installed here), but its row maps and
pooling arithmetic are pure torch. This script takes ``MiniMaxH3TokenReduction``, ``reduced_token_width``,
``build_token_reduction``, ``pool_token_pairs`` and ``expand_token_pairs`` from the file's syntax tree unchanged and
runs them with torch on the CPU on the seeded inputs of ``cases.REDUCTION_CASES`` (a stand-in schedule object carries
begin, end and update_scale). The reduced stream the expansion restores from is the pooled stream plus a seeded
update. Run in a checkout that has the reference source tree: ``python tests/golden/gen_reduction_golden.py``.
"""
from __future__ import annotations

import ast
import sys
import types
from dataclasses import dataclass
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from cases import REDUCTION_CASES, reduction_inputs  # noqa: E402

from oracle.ref_build.build_ref import reference_root  # noqa: E402

NAMES = {"MiniMaxH3TokenReduction", "reduced_token_width", "build_token_reduction", "pool_token_pairs",
         "expand_token_pairs"}


def reference_functions() -> dict:
    src = reference_root() / "fastvideo" / "models" / "dits" / "minimax_h3_token_reduction.py"
    tree = ast.parse(src.read_text())
    keep = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in NAMES]
    assert {n.name for n in keep} == NAMES
    module = types.ModuleType("reference_token_reduction")  # dataclass() looks its module up in sys.modules
    sys.modules[module.__name__] = module
    ns = module.__dict__
    ns.update({"torch": torch, "dataclass": dataclass})
    future = ast.ImportFrom("__future__", [ast.alias("annotations")], 0)
    mod = ast.fix_missing_locations(ast.Module(body=[future] + keep, type_ignores=[]))
    exec(compile(mod, str(src), "exec"), ns)
    return ns


def main() -> None:
    ns = reference_functions()
    out = {}
    for name, c in REDUCTION_CASES.items():
        d = reduction_inputs(c["grid"], c["video_start"], c["C"], c["seed"])
        sched = SimpleNamespace(begin=1, end=2, update_scale=c["scale"])
        plan = ns["build_token_reduction"](d["positions"], c["video_start"], c["grid"], sched)
        pooled = ns["pool_token_pairs"](d["x"], plan)
        reduced = (pooled.float() + d["delta"].float()).bfloat16()
        restored = ns["expand_token_pairs"](d["x"], reduced, pooled, plan)
        for k in ("first", "second", "parents", "pair_reduced_rows", "pair_rows"):
            out[f"{name}.{k}"] = getattr(plan, k).numpy()
        out[f"{name}.positions"] = plan.position_ids.numpy()
        out[f"{name}.pooled"] = pooled[0].view(torch.int16).numpy()
        out[f"{name}.reduced"] = reduced[0].view(torch.int16).numpy()
        out[f"{name}.restored"] = restored[0].view(torch.int16).numpy()
    np.savez_compressed(HERE / "reduction.npz", **out)
    print("wrote", HERE / "reduction.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
