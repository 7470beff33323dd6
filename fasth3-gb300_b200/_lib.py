"""ctypes binding of ``lib/libh3b.so`` (declared in ``include/h3b.h``).

There is no fallback: if the library is missing or does not load, every op raises. A nonzero return code from the
library becomes ``RuntimeError(h3b_last_error())``, the way the reference's ``TORCH_CHECK`` failures surface.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libh3b.so"

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
F32 = ctypes.c_float
SZ = ctypes.c_size_t


class VsaArgs(ctypes.Structure):
    """Mirror of ``h3b_vsa_args``."""
    _fields_ = [
        ("q", P), ("k", P), ("v", P), ("out", P), ("lse", P), ("idx", P), ("num", P), ("vbs_q", P), ("vbs_kv", P),
        ("qs", P), ("ks", P), ("vs", P), ("vs_head", P), ("qk_coef", F32), ("heads", I32), ("n_q_ext", I32),
        ("n_kv", I32), ("idx_ld", I32), ("q_scale_ld", I32), ("kv_scale_ld", I32), ("rows_chunk_q", I64),
        ("rows_chunk_kv", I64), ("chunks_q", I32), ("chunks_kv", I32), ("qk_int8", I32),
    ]


class PeerCopy(ctypes.Structure):
    """Mirror of ``h3b_peer_copy``."""
    _fields_ = [("dst", P), ("src", P), ("dpitch", SZ), ("spitch", SZ), ("width", SZ), ("height", SZ)]


PEER_PUT_MAX_COPIES, PEER_PUT_MAX_FLAGS = 64, 16


class Epilogue(ctypes.Structure):
    """Mirror of ``h3b_epilogue``."""
    _fields_ = [
        ("alpha", F32),
        ("alpha_dev", P),
        ("row_scale", P),
        ("col_scale", P),
        ("col_scale_scalar", I32),
        ("bias", P),
        ("act", I32),
        ("residual", P),
        ("ldr", I64),
        ("gate", P),
        ("D", P),
        ("ldd", I64),
    ]


# name -> argtypes (restype is int unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "h3b_last_error": [],
    "h3b_version": [],
    "h3b_resid_norm_quant": [P, P, P, P, I64, P, I32, P, P, P, I64, P, P, P, P, F32, I64, I32, P],
    "h3b_quant_fp8_rows": [P, I64, I64, I32, P, P, P],
    "h3b_amax_bf16": [P, I64, I64, I32, P, P],
    "h3b_quant_nvfp4_tensor": [P, I64, I64, I32, P, P, P, P, P],
    "h3b_quant_nvfp4_workspace_bytes": [],
    "h3b_quant_nvfp4": [P, I64, I64, I32, P, P, P, P, P],
    "h3b_quant_nvfp4_noalloc": [P, I64, I64, I32, P, P, P, P],
    "h3b_quant_nvfp4_rows": [P, I64, I64, I32, P, P, P, P],
    "h3b_pack_weight_fp8": [P, I64, I32, I32, P, P, P, P],
    "h3b_pack_weight_nvfp4": [P, I64, I32, P, P, P, P, P],
    "h3b_quant_fp8_on_grid": [P, I64, I32, P, I32, P, P, P, P],
    "h3b_pool_pairs": [P, P, P, I64, I32, P, P, P],
    "h3b_expand_pairs": [P, I64, P, P, P, P, I32, F32, P],
    "h3b_gemm_fp8": [P, P, I64, I64, I64, ctypes.POINTER(Epilogue), P],
    "h3b_gemm_nvfp4": [P, P, P, P, I64, I64, I64, ctypes.POINTER(Epilogue), P],
    "h3b_gemm_nvfp4_requant": [P, P, P, P, I64, I64, I64, ctypes.POINTER(Epilogue), P, P, P, P],
    "h3b_qkv_prologue8": [P, P, P, I64, P, P, P, P, P, P, P, F32, F32, P, P, P, P, P, P, P, P, P, P, I32, I64, I32,
                          I32, F32, P],
    "h3b_qkv_prologue8_qk_int8": [P, P, P, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I32, I64, I32, I32,
                                  F32, P],
    "h3b_vsa_tile_quant": [P, P, P, I32, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, I64, I32, I32, P],
    "h3b_head_tile_quant": [P, I64, P, P, P, P, P, P, P, I32, I64, I32, I32, F32, P],
    "h3b_vsa_fp8": [P, P, P, P, P, P, P, P, P, P, F32, P, P, I32, I32, I32, I64, P],
    "h3b_vsa_status": [ctypes.POINTER(I32), I32],
    "h3b_vsa_fp8_ex": [ctypes.POINTER(VsaArgs), P],
    "h3b_vsa_fp8_ex_v16": [ctypes.POINTER(VsaArgs), P],
    "h3b_vsa_pair": [ctypes.POINTER(VsaArgs), P, P],
    "h3b_vsa_pair_v16": [ctypes.POINTER(VsaArgs), P, P],
    "h3b_vsa_fp8_shared": [ctypes.POINTER(VsaArgs), P],
    "h3b_vsa_fp8_shared_v16": [ctypes.POINTER(VsaArgs), P],
    "h3b_vsa_fp8_ws": [ctypes.POINTER(VsaArgs), P],
    "h3b_qkv_prologue8_tiles": [P, P, P, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I32, I64, I32, I32,
                                F32, I32, P],
    "h3b_vsa_tile_quant_v16": [P, P, P, I32, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, I64, I32, I32, P],
    "h3b_head_tile_quant_v16": [P, I64, P, P, P, P, P, P, P, I32, I64, I32, I32, F32, P],
    "h3b_tile_scores": [P, P, I32, I32, F32, P, P],
    "h3b_topk_rows": [P, I32, I32, I32, I32, I32, P, P, P, P, P, I32, P],
    "h3b_topk_pairs": [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P],
    "h3b_compressed_branch": [P, P, I32, I32, P, P],
    "h3b_attn_gate_quant": [P, P, P, P, P, I64, I32, I32, P, P, P, I64, I32, P, P, P, I32, P, P],
    "h3b_device_status": [ctypes.POINTER(I32)],
    "h3b_reset_device_status": [],
    "h3b_status_async": [P, I32, P],
    "h3b_peer_alloc": [I32, SZ, ctypes.POINTER(P)],
    "h3b_peer_free": [P],
    "h3b_peer_export": [P, P],
    "h3b_peer_open": [P, ctypes.POINTER(P)],
    "h3b_peer_close": [P],
    "h3b_peer_copy2d": [P, SZ, P, SZ, SZ, SZ, P],
    "h3b_peer_signal": [P, ctypes.c_uint32, P],
    "h3b_peer_wait": [P, I32, ctypes.c_uint32, ctypes.c_uint64, P],
    "h3b_peer_put": [ctypes.POINTER(PeerCopy), I32, ctypes.POINTER(P), I32, ctypes.c_uint32, P, P],
    "h3b_selftest_wait_timeout": [ctypes.c_uint64, P],
}
_RESTYPES = {"h3b_last_error": ctypes.c_char_p, "h3b_version": ctypes.c_char_p,
             "h3b_quant_nvfp4_workspace_bytes": SZ}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library, with argument types set. Raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"h3b: {LIB_PATH} is missing; build it with `python fasth3-gb300_b200/build.py` "
                               "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().h3b_last_error().decode(errors="replace")
        raise RuntimeError(f"h3b error {rc}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
