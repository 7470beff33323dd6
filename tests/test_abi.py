"""The C-ABI library loads here (no GPU) and exports every entry point include/h3b.h declares; argument checks
reject bad calls with H3B_EINVAL and a message before any CUDA work."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "h3b.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(h3b):
    lib = h3b.lib()
    names = declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_the_header(h3b):
    from fasth3_b200._lib import SIGNATURES
    assert set(declared()) <= set(SIGNATURES), set(declared()) - set(SIGNATURES)


def test_version(h3b):
    assert b"sm_100a" in h3b.lib().h3b_version()


def _err(lib):
    return lib.h3b_last_error().decode()


@pytest.mark.parametrize("case", ["null_x", "bad_width", "bad_norm"])
def test_resid_norm_quant_rejects(h3b, case):
    lib = h3b.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails its argument checks first
    args = dict(x=fake, C=5120, norm=1)
    if case == "null_x":
        args["x"] = None
    elif case == "bad_width":
        args["C"] = 5000
    else:
        args["norm"] = 7
    rc = lib.h3b_resid_norm_quant(args["x"], None, None, None, 0, None, args["norm"], fake, fake, fake, 0, fake, fake,
                                  None, fake, 1e-5, 4, args["C"], None)
    assert rc == 1 and _err(lib)


def test_gemm_rejects_bad_k(h3b):
    from fasth3_b200._lib import Epilogue
    lib = h3b.lib()
    e = Epilogue()
    e.D = 256
    e.ldd = 256
    rc = lib.h3b_gemm_fp8(ctypes.c_void_p(256), ctypes.c_void_p(256), 128, 256, 100, ctypes.byref(e), None)
    assert rc == 1 and "multiple of 128" in _err(lib)
    rc = lib.h3b_gemm_nvfp4(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256),
                            128, 256, 128, ctypes.byref(e), None)
    assert rc == 1 and "multiple of 256" in _err(lib)


def test_nvfp4_needs_aligned_workspace(h3b):
    lib = h3b.lib()
    rc = lib.h3b_quant_nvfp4(ctypes.c_void_p(256), 64, 4, 64, ctypes.c_void_p(256), ctypes.c_void_p(256),
                             ctypes.c_void_p(256), ctypes.c_void_p(258), None)
    assert rc == 1 and "workspace" in _err(lib)


def test_ops_refuse_cpu_tensors(ops):
    import torch
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quant_fp8_rows(x, torch.zeros(4, 64, dtype=torch.uint8), torch.zeros(4))


def test_peer_put_rejects(h3b):
    """h3b_peer_put checks its arguments on the host before any launch: unaligned widths, too many copies or flags,
    a missing counter."""
    from fasth3_b200._lib import PEER_PUT_MAX_COPIES, PeerCopy
    lib = h3b.lib()
    fake = 1 << 20  # never dereferenced: every call below fails its checks first
    ok = PeerCopy(fake, fake, 64, 64, 32, 2)
    odd = PeerCopy(fake, fake, 64, 64, 30, 2)
    flags = (ctypes.c_void_p * 1)(fake)
    cases = [((PeerCopy * 1)(odd), 1, flags, 1, fake, "multiples of 4"),
             ((PeerCopy * 1)(ok), PEER_PUT_MAX_COPIES + 1, flags, 1, fake, "copies"),
             ((PeerCopy * 1)(ok), 1, flags, 17, fake, "flags"),
             ((PeerCopy * 1)(ok), 1, flags, 1, None, "counter"),
             ((PeerCopy * 1)(PeerCopy(fake, fake, 16, 64, 32, 2)), 1, flags, 1, fake, "pitch")]
    for arr, n, fl, nf, counter, what in cases:
        assert lib.h3b_peer_put(arr, n, fl, nf, 1, counter, None) == 1, what
        assert what in _err(lib), (what, _err(lib))
