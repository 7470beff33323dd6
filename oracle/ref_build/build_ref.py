"""TEST INFRASTRUCTURE ONLY: builds ``oracle/_ref/h3ref.so`` from the reference's ``h3fast.cu`` (read in place under
the reference checkout, never copied) plus ``h3ref_harness.cu``, for sm_100a, with the reference's own nvcc flags
(``-O3 --use_fast_math -std=c++17``, fastvideo/models/dits/h3fast/__init__.py:42) except the architecture.

This is this repository's recipe, not the reference's build system: nvcc is driven through torch's extension builder
because the reference TU is a torch extension. The output lands only in ``oracle/_ref/`` (git-ignored; it travels to
the GPU box with the snapshot, where ``load()`` imports the prebuilt file without the reference sources).

Run: ``python oracle/ref_build/build_ref.py`` (needs the reference source tree: $H3_REFERENCE, else the default
of ``reference_root()``).
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref"
SO = OUT / "h3ref.so"
REF_DIR_REL = Path("fastvideo/models/dits/h3fast")


def reference_root() -> Path:
    return Path(os.environ.get("H3_REFERENCE", "/root/reference"))


def build_if_possible(verbose: bool = False) -> Path | None:
    src_dir = reference_root() / REF_DIR_REL
    if not (src_dir / "h3fast.cu").exists():
        if verbose:
            print("h3ref: reference sources absent; using the prebuilt oracle/_ref (if any)")
        return SO if SO.exists() else None
    harness = HERE / "h3ref_harness.cu"
    if SO.exists() and SO.stat().st_mtime > max(harness.stat().st_mtime, (src_dir / "h3fast.cu").stat().st_mtime):
        return SO
    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    load(name="h3ref", sources=[str(harness)], build_directory=str(OUT), extra_include_paths=[str(src_dir)],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode=arch=compute_100a,code=sm_100a", "-std=c++17"],
         verbose=verbose, is_python_module=False)
    if verbose:
        print(f"h3ref: built {SO}")
    return SO


_mod = None
_cdll = None


def load():
    """(pybind module with the reference ops, ctypes handle with the harness launchers) from the prebuilt .so,
    or (None, None) if it was not built."""
    global _mod, _cdll
    if _mod is None and SO.exists():
        import torch  # noqa: F401  (libtorch must be loaded first)
        spec = importlib.util.spec_from_file_location("h3ref", SO)
        _mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(_mod)
        _cdll = ctypes.CDLL(str(SO))
        P, I64, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        _cdll.h3ref_resid_norm_quant_5120.argtypes = [P, P, P, P, I64, P, P, P, P, I64, P, P, P, P, F, I64, P]
        _cdll.h3ref_quant_nvfp4_tensor.argtypes = [P, I64, ctypes.c_int, P, P, P, P, P]
        _cdll.h3ref_attn_gate_quant_5120.argtypes = [P, P, P, P, P, I64, ctypes.c_int, ctypes.c_int, P, P, P, I64, P]
    return _mod, _cdll


if __name__ == "__main__":
    path = build_if_possible(verbose=True)
    sys.exit(0 if path else 1)
