"""Generates ``tests/golden/layout_from_metadata.npz`` from the REFERENCE's own ``H3FastRunner._get_layout``.

The method lives in fastvideo/models/dits/h3fast/__init__.py (:183-260); the module imports FastVideo, which is not
installed here. This script takes the ``_Layout`` dataclass and the ``_get_layout`` function from the file's syntax
tree unchanged and runs them with torch on the CPU, on a stand-in runner (the attributes the method reads: heads,
head_dim, hidden, ffn, the FP8/NVFP4 switches, the dense-prefix options) and on FastVideo-style metadata from
``layout.vsa_metadata`` for the latent grids and prefix lengths of ``cases.LAYOUT_CASES``. The fixture holds the
reference's row maps (perm, inv, slot, tile_row0, vbs, vbs_ext), tile counts and dense-prefix row count.
Run in a checkout that has the reference source tree: ``python tests/golden/gen_layout_golden.py [REFERENCE_DIR]``.
"""
from __future__ import annotations

import ast
import dataclasses
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from cases import LAYOUT_CASES  # noqa: E402

from oracle.ref_build.build_ref import reference_root  # noqa: E402


def reference_get_layout(root: str | None = None):
    ref = reference_root(root)
    if ref is None:
        raise SystemExit("the reference source tree was not found (argument, $H3_REFERENCE or ../reference)")
    src = ref / "fastvideo" / "models" / "dits" / "h3fast" / "__init__.py"
    tree = ast.parse(src.read_text())
    keep = []
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and node.name == "_Layout":
            keep.append(node)
        if isinstance(node, ast.ClassDef) and node.name == "H3FastRunner":
            keep += [f for f in node.body if isinstance(f, ast.FunctionDef) and f.name == "_get_layout"]
    ns = {"torch": torch, "dataclass": dataclasses.dataclass, "Any": object, "_FP8": torch.float8_e4m3fn}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(src), "exec"), ns)
    return ns["_get_layout"]


def main() -> None:
    get_layout = reference_get_layout(sys.argv[1] if len(sys.argv) > 1 else None)
    import __graft_entry__
    layout = __graft_entry__.load_package().layout
    out = {}
    for name, c in LAYOUT_CASES.items():
        m = layout.vsa_metadata(tuple(c["grid"]), c["prefix"])
        rows = m["untile_combined_index"].numel()
        meta = types.SimpleNamespace(untile_combined_index=m["untile_combined_index"],
                                     variable_block_sizes=m["variable_block_sizes"], tile_elems=64,
                                     num_prefix_tiles=m["num_prefix_tiles"])
        runner = types.SimpleNamespace(heads=2, head_dim=128, hidden=256, ffn=512, fp4=False, fp8_attn=True,
                                       qk16=False, pair128=False, dense_prefix="fp8", dense_prefix_min_rows=0,
                                       layouts={})
        rotary = (torch.zeros(rows, 96), torch.zeros(rows, 96))
        L = get_layout(runner, rows, torch.device("cpu"), meta, rotary, torch.zeros(rows, dtype=torch.int64))
        for key in ("perm", "inv", "slot", "tile_row0", "vbs", "vbs_ext"):
            out[f"{name}.{key}"] = getattr(L, key).numpy()
        out[f"{name}.n_tiles"] = np.int64(L.n_tiles)
        out[f"{name}.n_ext"] = np.int64(L.n_ext)
        out[f"{name}.n_pre"] = np.int64(L.n_pre)
    np.savez_compressed(HERE / "layout_from_metadata.npz", **out)
    print("wrote", HERE / "layout_from_metadata.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
