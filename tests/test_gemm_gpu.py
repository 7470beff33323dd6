"""GPU parity of the tcgen05 GEMMs and their fused epilogues.

Oracle: the reference's dequantize-then-matmul in fp32 (its CPU torch path), the epilogue applied in fp32, then
rounded to bf16 like the kernel's output. Tolerance: rel-Frobenius <= 1e-3 for both FP8 and NVFP4 (the north star
allows 2e-2 for NVFP4; operands are the same quantized codes on both sides, so only the accumulation order and the
bf16 output rounding differ).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import outlier_matrix
from oracle import quant as oq
from test_oracle import assert_codes

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def gelu_tanh(v: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.gelu(v, approximate="tanh")


def epilogue_ref(acc, alpha=1.0, row=None, col=None, bias=None, act=None, residual=None, gate=None):
    v = acc * alpha
    if row is not None:
        v = v * row[:, None]
    if col is not None:
        v = v * (col if col.numel() > 1 else col.reshape(1))[None, :]
    if bias is not None:
        v = v + bias.float()[None, :]
    if act == "gelu_tanh":
        v = gelu_tanh(v)
    if residual is not None:
        v = residual.float() + gate.float()[None, :] * v
    return v.bfloat16().float()


def fp8_operands(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn(N, K, generator=g) * 4).clamp(-448, 448).to(torch.float8_e4m3fn)
    return a, w


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (2048, 3072, 3072), (300, 512, 256), (128, 272, 384),
                                   (1, 16, 128), (777, 1040, 640)])
def test_fp8_gemm_plain(ops, M, N, K):
    a, w = fp8_operands(M, N, K, seed=M + N + K)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_fp8(a.to(DEV), w.to(DEV), out)
    torch.cuda.synchronize()
    ref = epilogue_ref(a.float() @ w.float().T)
    assert rel(out.cpu().float(), ref) < TOL


@pytest.mark.parametrize("epi", ["scales_bias", "gelu", "residual", "all"])
def test_fp8_gemm_epilogues(ops, epi):
    M, N, K = 640, 768, 512
    a, w = fp8_operands(M, N, K, seed=3)
    g = torch.Generator().manual_seed(4)
    row = torch.rand(M, generator=g) + 0.5
    col = torch.rand(N, generator=g) * 0.01
    bias = torch.randn(N, generator=g).bfloat16()
    res = torch.randn(M, N, generator=g).bfloat16()
    gate = (torch.randn(N, generator=g) * 0.5).bfloat16()
    kw = {}
    if epi in ("scales_bias", "all", "gelu"):
        kw.update(row=row, col=col)
    if epi in ("scales_bias", "all"):
        kw.update(bias=bias)
    if epi in ("gelu", "all"):
        kw.update(act="gelu_tanh")
    if epi in ("residual", "all"):
        kw.update(residual=res, gate=gate)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    d = lambda t: None if t is None else t.to(DEV)  # noqa: E731
    ops.gemm_fp8(a.to(DEV), w.to(DEV), out, scale_a=d(kw.get("row")), scale_b=d(kw.get("col")),
                 bias=d(kw.get("bias")), act=kw.get("act"), residual=d(kw.get("residual")), gate=d(kw.get("gate")))
    torch.cuda.synchronize()
    ref = epilogue_ref(a.float() @ w.float().T, **kw)
    assert rel(out.cpu().float(), ref) < TOL, epi


def test_fp8_gemm_residual_in_place(ops):
    # the gated residual may write over its own residual input (the block's x <- x + gate * proj(y) update)
    M, N, K = 256, 512, 256
    a, w = fp8_operands(M, N, K, seed=8)
    res = torch.randn(M, N, generator=torch.Generator().manual_seed(9)).bfloat16()
    gate = torch.full((N,), 0.25).bfloat16()
    x = res.to(DEV).clone()
    ops.gemm_fp8(a.to(DEV), w.to(DEV), x, residual=x, gate=gate.to(DEV))
    torch.cuda.synchronize()
    ref = epilogue_ref(a.float() @ w.float().T, residual=res, gate=gate)
    assert rel(x.cpu().float(), ref) < TOL


def test_fp8_linear_config1_end_to_end(ops):
    """per-token e4m3 activations, per-channel e4m3 weights, Y = dequant(Xq) dequant(Wq)^T + 0."""
    M, N, K = 2048, 3072, 3072
    x = outlier_matrix(M, K, 0, 0.01, 20.0)
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(1)) * 0.02).bfloat16()
    bias = torch.zeros(N, dtype=torch.bfloat16)
    xd = x.to(DEV)
    q = torch.empty(M, K, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(M, device=DEV)
    ops.quant_fp8_rows(xd, q, s)
    wq, ws = ops.quantize_fp8_weight(w.to(DEV), "channel")
    y = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_fp8(q, wq, y, scale_a=s, scale_b=ws, bias=bias.to(DEV))
    torch.cuda.synchronize()
    # the activation codes agree with the CPU oracle outside its ambiguity window and the weight bytes exactly ...
    codes, s_ref, amb = oq.quant_fp8_rows(x.float().numpy())
    assert_codes(q.view(torch.uint8).cpu().numpy(), codes, amb, "config 1 activation codes")
    np.testing.assert_allclose(s.cpu().numpy(), s_ref, rtol=2e-7)
    rq, rs = oq.quantize_fp8_weight(w, "channel")
    assert torch.equal(wq.cpu().view(torch.uint8), rq.view(torch.uint8)) and torch.equal(ws.cpu(), rs)
    # ... and the GEMM equals dequantize-then-matmul in fp32 of those operands
    xq = q.cpu().float() * s.cpu()[:, None]
    ref = (xq @ (rq.float() * rs[:, None]).T + bias.float()).bfloat16().float()
    assert rel(y.cpu().float(), ref) < TOL
    # and the linear as a whole stays at FP8's error level against the unquantized product
    assert rel(y.cpu().float(), x.float() @ w.float().T) < 0.05


def nvfp4_operands(ops, M, N, K, seed):
    x = outlier_matrix(M, K, seed, 0.005, 30.0)
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(seed + 1)) * 0.02).bfloat16()
    qa = torch.empty(M, K // 2, device=DEV, dtype=torch.uint8)
    sfa = torch.empty(ops.sf_rows(M), K // 16, device=DEV, dtype=torch.uint8)
    sa = torch.empty(1, device=DEV)
    ops.quant_nvfp4(x.to(DEV), qa, sfa, sa, torch.empty(256, device=DEV, dtype=torch.uint8))
    qw, sfw, sw = ops.pack_nvfp4_weight(w.to(DEV))
    torch.cuda.synchronize()
    a_deq = torch.from_numpy(oq.dequant_nvfp4(qa.cpu().numpy(), sfa.cpu().numpy(), M, K, 1.0))
    w_deq = torch.from_numpy(oq.dequant_nvfp4(qw.cpu().numpy(), sfw.cpu().numpy(), N, K, 1.0))
    return (qa, sfa, sa, qw, sfw, sw), a_deq, w_deq, x, w


@pytest.mark.parametrize("M,N,K", [(128, 192, 256), (256, 384, 512), (300, 400, 768), (1000, 13824, 5120),
                                   (129, 5120, 1024)])
def test_nvfp4_gemm(ops, M, N, K):
    (qa, sfa, sa, qw, sfw, sw), a_deq, w_deq, _, _ = nvfp4_operands(ops, M, N, K, seed=M + K)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_nvfp4(qa, sfa, qw, sfw, out, alpha_dev=sa, scale_b=sw)
    torch.cuda.synchronize()
    ref = epilogue_ref(a_deq @ w_deq.T, alpha=sa.item() * sw.item())
    assert rel(out.cpu().float(), ref) < TOL


def test_nvfp4_gemm_epilogue_gelu_residual(ops):
    M, N, K = 384, 576, 512
    (qa, sfa, sa, qw, sfw, sw), a_deq, w_deq, _, _ = nvfp4_operands(ops, M, N, K, seed=21)
    g = torch.Generator().manual_seed(22)
    bias = torch.randn(N, generator=g).bfloat16()
    res = torch.randn(M, N, generator=g).bfloat16()
    gate = torch.randn(N, generator=g).bfloat16()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_nvfp4(qa, sfa, qw, sfw, out, alpha_dev=sa, scale_b=sw, bias=bias.to(DEV), act="gelu_tanh",
                   residual=res.to(DEV), gate=gate.to(DEV))
    torch.cuda.synchronize()
    ref = epilogue_ref(a_deq @ w_deq.T, alpha=sa.item() * sw.item(), bias=bias, act="gelu_tanh", residual=res,
                       gate=gate)
    assert rel(out.cpu().float(), ref) < TOL


@pytest.mark.parametrize("M,N,K", [(300, 400, 512), (1000, 5120, 1024)])
def test_nvfp4_gemm_residual_in_place(ops, M, N, K):
    """x <- x + gate * (A W^T) with the output over its own residual (the block's update): the epilogue reads each
    residual block by TMA before the same block is stored; ragged M and N exercise the clipped edge boxes."""
    (qa, sfa, sa, qw, sfw, sw), a_deq, w_deq, _, _ = nvfp4_operands(ops, M, N, K, seed=M + N)
    g = torch.Generator().manual_seed(23)
    res = torch.randn(M, N, generator=g).bfloat16()
    gate = torch.randn(N, generator=g).bfloat16()
    x = res.to(DEV).clone()
    ops.gemm_nvfp4(qa, sfa, qw, sfw, x, alpha_dev=sa, scale_b=sw, residual=x, gate=gate.to(DEV))
    torch.cuda.synchronize()
    ref = epilogue_ref(a_deq @ w_deq.T, alpha=sa.item() * sw.item(), residual=res, gate=gate)
    assert rel(x.cpu().float(), ref) < TOL


@pytest.mark.parametrize("M,N,K,headroom", [(300, 384, 512, 2.0), (4099, 1536, 1024, 2.0), (1000, 13824, 5120, 2.0),
                                            (257, 576, 512, 0.25)])
def test_nvfp4_requant_epilogue_vs_oracle(ops, M, N, K, headroom):
    """The fc_in form: GEMM + bias + GELU-tanh with the output re-quantized to NVFP4 in the epilogue under a fixed
    global scale s. The codes and block scales equal the oracle's block math applied to the bf16 output of the same
    GEMM (h3b_gemm_nvfp4 with the same epilogue) under gs = 1/s; headroom 0.25 puts s below amax/2688, so the largest
    blocks saturate (scale 448, codes +-6) in both."""
    (qa, sfa, sa, qw, sfw, sw), _, _, _, _ = nvfp4_operands(ops, M, N, K, seed=M + 3 * N)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(M)) * 0.1).bfloat16().to(DEV)
    u = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_nvfp4(qa, sfa, qw, sfw, u, alpha_dev=sa, scale_b=sw, bias=bias, act="gelu_tanh")
    s = (u.float().abs().amax() * headroom / 2688.0).reshape(1).contiguous()
    q = torch.full((M, N // 2), 0xEE, device=DEV, dtype=torch.uint8)
    q_sf = torch.zeros(ops.sf_rows(M), N // 16, device=DEV, dtype=torch.uint8)
    ops.gemm_nvfp4_requant(qa, sfa, qw, sfw, q, q_sf, s, alpha_dev=sa, scale_b=sw, bias=bias, act="gelu_tanh")
    ops.check_status()
    uf = u.float().cpu().numpy()
    gs = np.float32(np.float32(1.0) / np.float32(s.item()))
    codes, bits, _, _ = oq.nvfp4_blocks(uf, gs)
    if headroom < 1:
        assert (bits == 0x7E).any(), "the small global scale should saturate some block scales"
    # the epilogue divides and multiplies with IEEE rounding (no fast math in the GEMM), like the oracle: bit-exact
    np.testing.assert_array_equal(oq.unswizzle_sf(q_sf.cpu().numpy(), M, N // 16), bits)
    np.testing.assert_array_equal(oq.unpack_nibbles(q.cpu().numpy()), codes)
    # and the next GEMM reading q with alpha = s reproduces u to NVFP4's error level
    deq = oq.dequant_nvfp4(q.cpu().numpy(), q_sf.cpu().numpy(), M, N, s.item())
    if headroom >= 1:
        assert rel(torch.from_numpy(deq), u.float().cpu()) < 0.12


def test_nvfp4_config2_full_size_sampled_rows(ops):
    """BASELINE config 2 at full size (32768 x 13824 x 5120): the whole GEMM runs on the GPU; 64 sampled rows are
    checked against the dequantize-then-matmul oracle, plus a checksum of every row against the oracle's row sums."""
    M, N, K = 32768, 13824, 5120
    x = outlier_matrix(M, K, 2, 0.005, 30.0)
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(3)) * 0.02).bfloat16()
    qa = torch.empty(M, K // 2, device=DEV, dtype=torch.uint8)
    sfa = torch.empty(ops.sf_rows(M), K // 16, device=DEV, dtype=torch.uint8)
    sa = torch.empty(1, device=DEV)
    ops.quant_nvfp4(x.to(DEV), qa, sfa, sa, torch.empty(256, device=DEV, dtype=torch.uint8))
    qw, sfw, sw = ops.pack_nvfp4_weight(w.to(DEV))
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops.gemm_nvfp4(qa, sfa, qw, sfw, out, alpha_dev=sa, scale_b=sw)
    torch.cuda.synchronize()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(4))[:64]
    a_deq = torch.from_numpy(oq.dequant_nvfp4(qa[rows].cpu().numpy(), _sf_rows(sfa, rows, K), 64, K, 1.0))
    w_deq = torch.from_numpy(oq.dequant_nvfp4(qw.cpu().numpy(), sfw.cpu().numpy(), N, K, 1.0))
    ref = epilogue_ref(a_deq @ w_deq.T, alpha=sa.item() * sw.item())
    assert rel(out[rows.to(DEV)].cpu().float(), ref) < TOL
    # linearity checksum over all rows: out @ 1 == A_deq @ (W_deq^T @ 1) * alpha (fp32, loose: bf16 rounding)
    wsum = (w_deq.sum(0) * sa.item() * sw.item()).to(DEV)
    a_all = _dequant_gpu(qa, sfa, M, K)
    want = a_all @ wsum
    got = out.float().sum(1)
    assert rel(got, want) < 5e-3


def _sf_rows(sfa: torch.Tensor, rows: torch.Tensor, K: int) -> np.ndarray:
    """The scale bytes of the selected rows, re-laid out as a dense 128x4 buffer for those rows."""
    full = sfa.cpu().numpy()
    n_all = full.shape[0]
    bits = oq.unswizzle_sf(full, n_all, K // 16)[rows.numpy()]
    return oq.swizzle_sf(bits)


def _dequant_gpu(q: torch.Tensor, sf: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """Dequantize NVFP4 on the GPU with plain torch ops (test-side reference only)."""
    lut = torch.tensor(oq.E2M1_VALUES, device=q.device)
    codes = torch.stack([q & 15, q >> 4], -1).reshape(rows, K)
    vals = lut[codes.long()].view(rows, K // 16, 16)
    r = torch.arange(rows, device=q.device)[:, None]
    c = torch.arange(K // 16, device=q.device)[None, :]
    off = (r >> 7) * (K // 64) * 512 + (c >> 2) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3)
    s = sf.reshape(-1)[off].view(torch.float8_e4m3fn).float()
    return (vals * s[..., None]).reshape(rows, K)


def test_bounded_wait_expires_with_status_and_context_survives(ops):
    """A wait that nothing completes gives up after its limit and reports H3B_ETIMEOUT through the status word, with
    no fault: the same context then runs a GEMM correctly and the status reads clean after a reset."""
    import time

    ops.reset_device_status()
    t0 = time.time()
    ops.selftest_wait_timeout(50_000_000)  # 50 ms
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert ops.device_status() == 3  # H3B_ETIMEOUT
    assert 0.04 < waited < 5.0
    ops.reset_device_status()
    assert ops.device_status() == 0
    g = torch.Generator().manual_seed(123)
    a = (torch.randn(256, 512, generator=g) * 4).to(torch.float8_e4m3fn).to(DEV)
    w = (torch.randn(384, 512, generator=g) * 4).to(torch.float8_e4m3fn).to(DEV)
    y = torch.empty(256, 384, device=DEV, dtype=torch.bfloat16)
    ops.gemm_fp8(a, w, y)
    torch.cuda.synchronize()
    ref = (a.float() @ w.float().t()).bfloat16().float()
    assert rel(y.float().cpu(), ref.cpu()) < TOL
    assert ops.device_status() == 0


def test_check_status_raises_after_an_expired_wait(ops):
    """ops.check_status (what the runner calls after each step) turns an expired wait into a RuntimeError, clears the
    word, and passes on the next check."""
    ops.check_status()
    ops.selftest_wait_timeout(20_000_000)  # 20 ms
    with pytest.raises(RuntimeError, match="ETIMEOUT"):
        ops.check_status()
    ops.check_status()
    assert ops.device_status() == 0


def test_exchange_wait_expires_raises_and_later_waits_skip(ops):
    """The peer transport's wait (h3b_peer_wait) on a flag that nothing sets gives up after its limit, sets the
    exchange status word (check_status raises "exchange waits"), makes the waits after it return at once instead of
    each waiting out its own limit, and the context stays usable; a flag that holds the epoch passes without waiting."""
    import time

    ops.check_status()
    flags = torch.zeros(4, device=DEV, dtype=torch.int32)
    t0 = time.time()
    ops.peer_wait(flags, 1, 200_000_000)  # 200 ms, nothing sets the flags
    for _ in range(5):  # skipped: the word is already set
        ops.peer_wait(flags, 1, 200_000_000)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert 0.15 < waited < 0.8, waited  # one limit, not six
    with pytest.raises(RuntimeError, match="exchange waits: H3B_ETIMEOUT"):
        ops.check_status()
    flags.fill_(7)
    ops.peer_wait(flags, 7, 30_000_000)   # reached
    ops.peer_wait(flags, 3, 30_000_000)   # passed long ago (wrap-around compare)
    torch.cuda.synchronize()
    ops.check_status()


@pytest.mark.parametrize("aligned", [True, False])
def test_peer_put_copies_then_raises_the_flags(ops, aligned):
    """h3b_peer_put (the SM form of the peer transport's small copies): 2D regions of several geometries land where
    cudaMemcpy2D would put them (16-byte units when every address, pitch and width allows, else 4-byte units), every
    flag holds the epoch afterwards, the counter is back at zero, and a bounded wait on the flags passes at once."""
    import ctypes

    from fasth3_b200._lib import PeerCopy, call
    g = torch.Generator(device=DEV).manual_seed(5)
    src = torch.randint(0, 2 ** 31 - 1, (3 << 20,), device=DEV, generator=g, dtype=torch.int32)
    dst = torch.zeros(4 << 20, device=DEV, dtype=torch.int32)
    want = dst.clone()
    sb, db = src.view(torch.uint8), want.view(torch.uint8)
    e = 0 if aligned else 4  # byte skew of every address, pitch and width
    geo = [(0, 4096, 0, 8192, 1008, 40), (64 << 10, 65536 + e, 1 << 20, 131072 + e, 64512 + e, 5),
           (2 << 20, 512 + e, 3 << 20, 768, 256 + e, 700), (1 << 10, 64, 6 << 20, 64, 16, 1), (0, 16, 0, 16, 0, 3)]
    copies = []
    for so, sp, do, dp, w, h in geo:
        so, do = so + e, do + e
        for row in range(h):
            db[do + row * dp:do + row * dp + w] = sb[so + row * sp:so + row * sp + w]
        copies.append(PeerCopy(dst.data_ptr() + do, src.data_ptr() + so, dp, sp, w, h))
    flags = torch.zeros(3, device=DEV, dtype=torch.int32)
    counter = torch.zeros(1, device=DEV, dtype=torch.int32)
    fl = (ctypes.c_void_p * 3)(*[flags.data_ptr() + 4 * i for i in range(3)])
    s = torch.cuda.current_stream().cuda_stream
    for epoch in (11, 12):
        call("h3b_peer_put", (PeerCopy * len(copies))(*copies), len(copies), fl, 3, epoch, counter.data_ptr(), s)
        ops.peer_wait(flags, epoch, 100_000_000)
        torch.cuda.synchronize()
        assert torch.equal(dst, want)
        assert flags.tolist() == [epoch] * 3 and int(counter) == 0
    ops.check_status()
