"""The allocation-free NVFP4 quantizer, for callers that cannot allocate device memory.

A host that passes the library only the buffers it already owns (a plugin inside an engine with a pre-planned memory
pool, or a foreign-language host with a fixed buffer set) cannot hand h3b_quant_nvfp4 a workspace it would have to
cudaMalloc mid-run; h3b_quant_nvfp4_noalloc keeps that scratch in a static device array instead. This test calls it
through the C ABI and checks it against h3b_quant_nvfp4 (the workspace version) bit for bit, on two calls in a row --
the second on a tensor with a smaller maximum, so a scratch word left over from the first call would show.

Named to be collected last, so a run that stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from cases import outlier_matrix

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _quantize_both(h3b, x):
    lib = h3b.lib()
    ops = h3b.ops
    rows, K = x.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for variant in ("workspace", "noalloc"):
        q = torch.full((rows, K // 2), 0x5A, device=DEV, dtype=torch.uint8)
        sf = torch.full((ops.sf_rows(rows), K // 16), 0xA5, device=DEV, dtype=torch.uint8)
        s = torch.full((1,), -1.0, device=DEV)
        if variant == "workspace":
            ws = torch.empty(ops.workspace_bytes(), device=DEV, dtype=torch.uint8)
            rc = lib.h3b_quant_nvfp4(x.data_ptr(), x.stride(0), rows, K, q.data_ptr(), sf.data_ptr(), s.data_ptr(),
                                     ws.data_ptr(), stream)
        else:
            rc = lib.h3b_quant_nvfp4_noalloc(x.data_ptr(), x.stride(0), rows, K, q.data_ptr(), sf.data_ptr(),
                                             s.data_ptr(), stream)
        assert rc == 0, lib.h3b_last_error().decode()
        outs.append((q, sf, s))
    torch.cuda.synchronize()
    return outs


def test_noalloc_matches_workspace_version_on_two_calls(h3b):
    first = outlier_matrix(1000, 5120, 31, 0.005, 30.0).to(DEV)          # amax ~ 130
    second = outlier_matrix(777, 3072, 32, 0.0, 1.0, std=0.5).to(DEV)     # amax ~ 2.5: smaller than the first
    for x in (first, second):
        (q0, sf0, s0), (q1, sf1, s1) = _quantize_both(h3b, x)
        assert torch.equal(s0, s1), (s0.item(), s1.item())
        assert torch.equal(q0, q1)
        assert torch.equal(sf0, sf1)


def test_noalloc_zero_rows_leaves_outputs(h3b):
    """rows == 0 is a valid call that writes nothing."""
    lib = h3b.lib()
    x = torch.zeros(1, 128, device=DEV, dtype=torch.bfloat16)
    q = torch.full((1, 64), 0x5A, device=DEV, dtype=torch.uint8)
    sf = torch.full((128, 8), 0xA5, device=DEV, dtype=torch.uint8)
    s = torch.full((1,), -1.0, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.h3b_quant_nvfp4_noalloc(x.data_ptr(), 128, 0, 128, q.data_ptr(), sf.data_ptr(), s.data_ptr(), stream)
    torch.cuda.synchronize()
    assert rc == 0, lib.h3b_last_error().decode()
    assert (q == 0x5A).all() and (sf == 0xA5).all() and s.item() == -1.0


def test_noalloc_rejects_bad_arguments(h3b):
    lib = h3b.lib()
    x = torch.zeros(4, 100, device=DEV, dtype=torch.bfloat16)  # K not a multiple of 64
    q = torch.zeros(4, 50, device=DEV, dtype=torch.uint8)
    rc = lib.h3b_quant_nvfp4_noalloc(x.data_ptr(), 100, 4, 100, q.data_ptr(), q.data_ptr(), q.data_ptr(), None)
    assert rc == 1 and "multiple of 64" in lib.h3b_last_error().decode()
