"""TEST INFRASTRUCTURE ONLY: builds ``oracle/_ref/h3ref.so`` from the reference's ``h3fast.cu`` (read in place under
the reference checkout, never copied) plus ``h3ref_harness.cu``, for sm_100a, with the reference's own nvcc flags
(``-O3 --use_fast_math -std=c++17``, fastvideo/models/dits/h3fast/__init__.py:42) except the architecture.

This is this repository's recipe, not the reference's build system: nvcc is driven through torch's extension builder
because the reference TU is a torch extension. The output lands only in ``oracle/_ref/`` (git-ignored; it travels to
the GPU box with the snapshot, where ``load()`` imports the prebuilt file without the reference sources).

Run: ``python oracle/ref_build/build_ref.py [REFERENCE_DIR]`` (the reference source tree: the argument, else
$H3_REFERENCE, else a checkout named ``reference`` beside this repository).
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


def reference_root(explicit: str | None = None) -> Path | None:
    """The reference checkout: ``explicit``, else $H3_REFERENCE, else a sibling directory ``reference`` of this
    repository (None when none of them holds the sources)."""
    for cand in (explicit, os.environ.get("H3_REFERENCE"), str(HERE.parents[2] / "reference")):
        if cand and (Path(cand) / REF_DIR_REL / "h3fast.cu").exists():
            return Path(cand)
    return None


def build_if_possible(verbose: bool = False, root: str | None = None) -> Path | None:
    ref = reference_root(root)
    if ref is None:
        if verbose:
            print("h3ref: reference sources absent; using the prebuilt oracle/_ref (if any)")
        return SO if SO.exists() else None
    src_dir = ref / REF_DIR_REL
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


ATTN_OUT = OUT / "attn16"
ATTN_SO = ATTN_OUT / "h3ref_attn16.so"


def build_attn16_if_possible(verbose: bool = False, root: str | None = None) -> Path | None:
    """The reference's BF16 VSA kernel (h3attn16.cu with VSA_LDRED off) as its own extension module, the timing bar
    for the FP8 attention. Output in oracle/_ref/attn16/."""
    ref = reference_root(root)
    if ref is None:
        return ATTN_SO if ATTN_SO.exists() else None
    src_dir = ref / REF_DIR_REL
    harness = HERE / "h3ref_attn16_harness.cu"
    deps = [harness, src_dir / "h3attn16.cu", src_dir / "vsa_bf16.cuh", src_dir / "vsa_bf16_launch.cuh"]
    if ATTN_SO.exists() and ATTN_SO.stat().st_mtime > max(p.stat().st_mtime for p in deps):
        return ATTN_SO
    ATTN_OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import CUDA_HOME
    from torch.utils.cpp_extension import load as load_ext
    try:
        load_ext(name="h3ref_attn16", sources=[str(harness)], build_directory=str(ATTN_OUT),
                 extra_include_paths=[str(src_dir)],
                 extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode=arch=compute_100a,code=sm_100a",
                                    "-std=c++17"],
                 extra_ldflags=[f"-L{CUDA_HOME}/lib64/stubs", "-lcuda"], verbose=verbose, is_python_module=False)
    except OSError:
        # built, but not loadable on a machine without the CUDA driver (it links libcuda); the GPU box loads it
        if not ATTN_SO.exists():
            raise
    if verbose:
        print(f"h3ref: built {ATTN_SO}")
    return ATTN_SO


_attn_mod = None


def load_attn16():
    """The pybind module holding the reference's BF16 VSA forward (``vsa_bf16``), or None if it was not built."""
    global _attn_mod
    if _attn_mod is None and ATTN_SO.exists():
        import torch  # noqa: F401  (libtorch must be loaded first)
        spec = importlib.util.spec_from_file_location("h3ref_attn16", ATTN_SO)
        _attn_mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(_attn_mod)
    return _attn_mod


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
    root = sys.argv[1] if len(sys.argv) > 1 else None
    path = build_if_possible(verbose=True, root=root)
    attn = build_attn16_if_possible(verbose=True, root=root)
    sys.exit(0 if path and attn else 1)
