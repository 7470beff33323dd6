"""Tensor-level ops over the h3b C ABI, with the reference extension's names and argument meaning.

Every op writes into caller-allocated buffers (the reference ops do the same, fastvideo/models/dits/h3fast/h3fast.cu:
831-1073), runs on the current CUDA stream and raises ``RuntimeError`` on a bad argument. CUDA tensors only: there is
no CPU path.
"""
from __future__ import annotations

import torch

from ._lib import Epilogue, call, lib

FP8 = torch.float8_e4m3fn
NORMS = {"none": 0, "rms": 1, "layer": 2}
ACTS = {None: 0, "none": 0, "gelu_tanh": 1}
GRAN = {"tensor": 0, "channel": 1}


def _p(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("h3b ops take CUDA tensors only (no CPU fallback)")
    return t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _contig(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def sf_rows(rows: int) -> int:
    """Rows of a block-scale buffer: padded to the 128-row atom."""
    return (rows + 127) // 128 * 128


# ------------------------------------------------------------------------------------------------- row quantizers
def resid_norm_quant(x: torch.Tensor, y: torch.Tensor | None, sy: torch.Tensor | None, gate: torch.Tensor | None,
                     idx: torch.Tensor | None, nw: torch.Tensor | None, shift: torch.Tensor | None,
                     scale: torch.Tensor | None, xo: torch.Tensor, h: torch.Tensor | None, hsf: torch.Tensor | None,
                     hs: torch.Tensor | None, eps: float, norm: str | None = None) -> None:
    """Gated residual and/or norm + adaLN modulate + FP8/NVFP4 row quantization (h3fast.cu:831-858 semantics).

    Passing no ``y`` skips the residual; passing no ``nw`` skips the norm unless ``norm="layer"`` (LayerNorm without
    affine parameters, which needs no weight). ``hsf`` given selects NVFP4 (``h`` then holds [rows, C/2] codes).
    """
    C = x.shape[-1]
    _contig(x, "x")
    rows = x.numel() // C
    if norm is None:
        norm = "rms" if nw is not None else "none"
    gate_ld = gate.stride(0) if gate is not None else 0
    tab_ld = scale.stride(0) if scale is not None else 0
    if idx is not None and idx.dtype != torch.int32:
        raise RuntimeError("idx must be int32")
    call("h3b_resid_norm_quant", _p(x), _p(y), _p(sy), _p(gate), gate_ld, _p(idx), NORMS[norm], _p(nw), _p(shift),
         _p(scale), tab_ld, _p(xo), _p(h), _p(hsf), _p(hs), float(eps), rows, C, _stream(x))


def quant_fp8_rows(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
    """Per-token FP8: s[r] = max(amax_r/448, 1/(448*512)), q = e4m3(x / s[r])."""
    K = x.shape[-1]
    rows = x.numel() // K
    call("h3b_quant_fp8_rows", _p(x), x.stride(-2) if x.dim() > 1 else K, rows, K, _p(q), _p(s), _stream(x))


def amax(x: torch.Tensor, out: torch.Tensor) -> None:
    """Folds max|x| into out[0] (atomic max; out must start at 0 or a partial maximum)."""
    K = x.shape[-1]
    call("h3b_amax_bf16", _p(x), x.stride(-2) if x.dim() > 1 else K, x.numel() // K, K, _p(out), _stream(x))


def quant_nvfp4_tensor(x: torch.Tensor, amax_dev: torch.Tensor, q: torch.Tensor, sf: torch.Tensor,
                       s_out: torch.Tensor) -> None:
    """NVFP4 with a per-tensor global scale from a device amax: s = max(amax/2688, 1e-12)."""
    K = x.shape[-1]
    call("h3b_quant_nvfp4_tensor", _p(x), x.stride(-2) if x.dim() > 1 else K, x.numel() // K, K, _p(amax_dev), _p(q),
         _p(sf), _p(s_out), _stream(x))


def quant_nvfp4_rows(x: torch.Tensor, q: torch.Tensor, sf: torch.Tensor, s_rows: torch.Tensor) -> None:
    """Per-row NVFP4 (global scale per row, s_rows[r] = max(amax_r/2688, 1e-12)) for any K multiple of 64."""
    K = x.shape[-1]
    call("h3b_quant_nvfp4_rows", _p(x), x.stride(-2) if x.dim() > 1 else K, x.numel() // K, K, _p(q), _p(sf),
         _p(s_rows), _stream(x))


def workspace_bytes() -> int:
    return int(lib().h3b_quant_nvfp4_workspace_bytes())


def quant_nvfp4(x: torch.Tensor, q: torch.Tensor, sf: torch.Tensor, s_out: torch.Tensor,
                workspace: torch.Tensor) -> None:
    """amax pass + per-tensor NVFP4 quantization in one call (workspace: >= workspace_bytes(), 256-aligned)."""
    K = x.shape[-1]
    call("h3b_quant_nvfp4", _p(x), x.stride(-2) if x.dim() > 1 else K, x.numel() // K, K, _p(q), _p(sf), _p(s_out),
         _p(workspace), _stream(x))


# ------------------------------------------------------------------------------------------------- token reduction
def pool_pairs(x: torch.Tensor, ia: torch.Tensor, ib: torch.Tensor, out: torch.Tensor,
               pooled: torch.Tensor | None = None) -> torch.Tensor:
    """``H3FastRunner._pool`` (fastvideo/models/dits/h3fast/__init__.py:280-285): ``out[r] = (x[ia[r]] + x[ib[r]]) / 2``
    in float32 for bf16 rows; ``pooled`` (optional) receives the same rows."""
    _contig(x, "x")
    _contig(out, "out")
    C = x.shape[-1]
    for t, n in ((ia, "ia"), (ib, "ib")):
        if t.dtype != torch.int32 or t.numel() != out.shape[0]:
            raise RuntimeError(f"{n} must be int32 with one entry per output row")
    call("h3b_pool_pairs", _p(x), _p(ia), _p(ib), out.shape[0], C, _p(out), _p(pooled), _stream(x))
    return out


def expand_pairs(x: torch.Tensor, xr: torch.Tensor, pooled: torch.Tensor, par: torch.Tensor, pair: torch.Tensor,
                 scale: float) -> torch.Tensor:
    """``H3FastRunner._expand`` (:287-293), in place on ``x``: a paired row becomes ``x + scale * (xr - pooled)`` of
    its reduced row ``par``, every other row takes ``xr[par]``."""
    _contig(x, "x")
    C = x.shape[-1]
    if par.dtype != torch.int32 or par.numel() != x.shape[0] or pair.numel() != x.shape[0]:
        raise RuntimeError("par (int32) and pair need one entry per row of x")
    if pair.dtype not in (torch.bool, torch.uint8) or not pair.is_contiguous():
        raise RuntimeError("pair must be a contiguous bool or uint8 mask")
    call("h3b_expand_pairs", _p(x), x.shape[0], _p(xr), _p(pooled), _p(par), _p(pair.view(torch.uint8) if pair.dtype == torch.bool else pair), C,
         float(scale), _stream(x))
    return x


# ------------------------------------------------------------------------------------------------- weight packing
def quantize_fp8_weight(weight: torch.Tensor, granularity: str = "tensor",
                        workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(fp8 weight, float32 scale)`` of a dense bf16 ``[out, in]`` weight; the same contract as
    ``quantize_fp8_weight`` (patches/fastvideo-a01c50a.patch:384-394). Allocates its outputs like the reference."""
    _contig(weight, "weight")
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("weight must be bf16")
    N, K = weight.shape
    wq = torch.empty(N, K, device=weight.device, dtype=FP8)
    ws = torch.empty(N if granularity == "channel" else 1, device=weight.device, dtype=torch.float32)
    if workspace is None and granularity == "tensor":
        workspace = torch.empty(256, device=weight.device, dtype=torch.uint8)
    call("h3b_pack_weight_fp8", _p(weight), N, K, GRAN[granularity], _p(wq), _p(ws), _p(workspace), _stream(weight))
    return wq, ws


def pack_nvfp4_weight(weight: torch.Tensor, workspace: torch.Tensor | None = None
                      ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(codes uint8 [N, K/2], block scales uint8 [pad128(N), K/16] in the 128x4 layout, fp32 [1] tensor scale)``."""
    _contig(weight, "weight")
    N, K = weight.shape
    wq = torch.empty(N, K // 2, device=weight.device, dtype=torch.uint8)
    wsf = torch.empty(sf_rows(N), K // 16, device=weight.device, dtype=torch.uint8)
    ws = torch.empty(1, device=weight.device, dtype=torch.float32)
    if workspace is None:
        workspace = torch.empty(256, device=weight.device, dtype=torch.uint8)
    call("h3b_pack_weight_nvfp4", _p(weight), N, K, _p(wq), _p(wsf), _p(ws), _p(workspace), _stream(weight))
    return wq, wsf, ws


def quant_fp8_on_grid(merged: torch.Tensor, base_scale: torch.Tensor, workspace: torch.Tensor | None = None
                      ) -> tuple[torch.Tensor, torch.Tensor]:
    """``_on_grid`` (fastvideo/models/dits/h3fast/__init__.py:82-92): the fp32 ``merged`` weight (a LoRA folded into
    the dense weight) in E4M3 on the base weight's grid ``base_scale`` (one float32 per output row, or one for the
    tensor). A row (or the tensor) whose amax exceeds 1.05 x 448 x its grid scale gets its own scale amax / 448.
    Returns ``(fp8 weight [N, K], float32 scale [N] or [1])``."""
    _contig(merged, "merged")
    if merged.dtype != torch.float32:
        raise RuntimeError("merged must be float32")
    N, K = merged.shape
    per_row = base_scale.numel() > 1
    if per_row and base_scale.numel() != N:
        raise RuntimeError(f"base_scale has {base_scale.numel()} entries for {N} rows")
    base = base_scale.reshape(-1).to(torch.float32).contiguous()
    wq = torch.empty(N, K, device=merged.device, dtype=FP8)
    ws = torch.empty(N if per_row else 1, device=merged.device, dtype=torch.float32)
    if workspace is None and not per_row:
        workspace = torch.empty(256, device=merged.device, dtype=torch.uint8)
    call("h3b_quant_fp8_on_grid", _p(merged), N, K, _p(base), int(per_row), _p(wq), _p(ws), _p(workspace),
         _stream(merged))
    return wq, ws


# ------------------------------------------------------------------------------------------------- GEMMs
def _epilogue(out: torch.Tensor | None, alpha: float, alpha_dev, row_scale, col_scale, bias, act, residual,
              gate) -> Epilogue:
    e = Epilogue()
    e.alpha = float(alpha)
    e.alpha_dev = _p(alpha_dev)
    e.row_scale = _p(row_scale)
    e.col_scale = _p(col_scale)
    e.col_scale_scalar = int(col_scale is not None and col_scale.numel() == 1)
    e.bias = _p(bias)
    e.act = ACTS[act]
    e.residual = _p(residual)
    e.ldr = residual.stride(0) if residual is not None else 0
    e.gate = _p(gate)
    e.D = _p(out)
    e.ldd = out.stride(0) if out is not None else 0
    return e


def gemm_fp8(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *, scale_a: torch.Tensor | None = None,
             scale_b: torch.Tensor | None = None, bias: torch.Tensor | None = None, act: str | None = None,
             residual: torch.Tensor | None = None, gate: torch.Tensor | None = None, alpha: float = 1.0,
             alpha_dev: torch.Tensor | None = None) -> torch.Tensor:
    """out = epilogue(a @ w^T) for e4m3 a [M, K], w [N, K]: the ``torch._scaled_mm(a, w.t(), scale_a, scale_b)``
    call of H3FastRunner._gemm (fastvideo/models/dits/h3fast/__init__.py:389) with the epilogue fused in."""
    _contig(a, "a")
    _contig(w, "w")
    M, K = a.shape
    N = w.shape[0]
    e = _epilogue(out, alpha, alpha_dev, scale_a, scale_b, bias, act, residual, gate)
    call("h3b_gemm_fp8", _p(a), _p(w), M, N, K, e, _stream(a))
    return out


def gemm_nvfp4(a: torch.Tensor, a_sf: torch.Tensor, w: torch.Tensor, w_sf: torch.Tensor, out: torch.Tensor, *,
               alpha: float = 1.0, alpha_dev: torch.Tensor | None = None, scale_a: torch.Tensor | None = None,
               scale_b: torch.Tensor | None = None, bias: torch.Tensor | None = None, act: str | None = None,
               residual: torch.Tensor | None = None, gate: torch.Tensor | None = None) -> torch.Tensor:
    """out = epilogue(alpha * sum e2m1(a) sfA e2m1(w) sfB) for packed a [M, K/2], w [N, K/2] and their 128x4 block
    scales: FlashInfer's ``mm_fp4(a, w.T, a_sf, w_sf.T, alpha, bf16, out, block_size=16)`` as called at
    fastvideo/models/dits/h3fast/__init__.py:402, with the epilogue fused in."""
    _contig(a, "a")
    _contig(w, "w")
    M, K = a.shape[0], a.shape[1] * 2
    N = w.shape[0]
    e = _epilogue(out, alpha, alpha_dev, scale_a, scale_b, bias, act, residual, gate)
    call("h3b_gemm_nvfp4", _p(a), _p(a_sf), _p(w), _p(w_sf), M, N, K, e, _stream(a))
    return out


def gemm_nvfp4_requant(a: torch.Tensor, a_sf: torch.Tensor, w: torch.Tensor, w_sf: torch.Tensor, q: torch.Tensor,
                       q_sf: torch.Tensor, q_scale: torch.Tensor, *, alpha: float = 1.0,
                       alpha_dev: torch.Tensor | None = None, scale_a: torch.Tensor | None = None,
                       scale_b: torch.Tensor | None = None, bias: torch.Tensor | None = None,
                       act: str | None = None) -> torch.Tensor:
    """gemm_nvfp4 whose epilogue writes the output re-quantized for the next NVFP4 GEMM: q [M, N/2] packed e2m1 and
    q_sf [sf_rows(M), N/16] block scales under the fixed global scale ``q_scale`` (a device float; the next GEMM takes
    it as its alpha). Replaces the bf16 store plus the separate per-row quantization pass of the reference's FFN
    (h3fast.cu:781-817) when a static global scale is acceptable."""
    _contig(a, "a")
    _contig(w, "w")
    M, K = a.shape[0], a.shape[1] * 2
    N = w.shape[0]
    if q.shape != (M, N // 2) or q.dtype != torch.uint8 or not q.is_contiguous():
        raise ValueError(f"q must be contiguous uint8 [{M}, {N // 2}]")
    if q_sf.shape != (sf_rows(M), N // 16) or q_sf.dtype != torch.uint8:
        raise ValueError(f"q_sf must be uint8 [{sf_rows(M)}, {N // 16}]")
    if q_scale.numel() != 1 or q_scale.dtype != torch.float32:
        raise ValueError("q_scale must be one float32 on the device")
    e = _epilogue(None, alpha, alpha_dev, scale_a, scale_b, bias, act, None, None)
    call("h3b_gemm_nvfp4_requant", _p(a), _p(a_sf), _p(w), _p(w_sf), M, N, K, e, _p(q), _p(q_sf), _p(q_scale),
         _stream(a))
    return q


def device_status() -> int:
    import ctypes
    v = ctypes.c_int(0)
    call("h3b_device_status", ctypes.byref(v))
    return int(v.value)


def reset_device_status() -> None:
    call("h3b_reset_device_status")


_STATUS_NAMES = {1: "H3B_EINVAL (a selection list longer than the attention kernel holds)",
                 3: "H3B_ETIMEOUT (a kernel's bounded wait expired)"}
_status_bufs: dict = {}


def check_status(device: torch.device | str | None = None) -> None:
    """Reads the kernels' device status words after everything enqueued so far on the current stream (one host sync)
    and raises ``RuntimeError`` if a GEMM, attention, row kernel or exchange wait reported a failure since the last check (the words are
    cleared by the read). The runner calls this once per step, after the step's last kernel."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    buf = _status_bufs.get(dev.index)
    if buf is None:
        buf = _status_bufs[dev.index] = torch.zeros(4, dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    call("h3b_status_async", buf.data_ptr(), 1, stream.cuda_stream)
    stream.synchronize()
    words = (("GEMM", int(buf[0])), ("attention", int(buf[1])), ("row kernels", int(buf[2])),
             ("exchange waits", int(buf[3])))
    if any(v for _, v in words):
        parts = [f"{who}: {_STATUS_NAMES.get(v, v)}" for who, v in words if v]
        raise RuntimeError("h3b device status after the step -- " + "; ".join(parts))


def peer_wait(flags: torch.Tensor, epoch: int, limit_ns: int = 0) -> None:
    """Bounded wait on the current stream until every int32 word of ``flags`` reaches ``epoch`` (h3b_peer_wait: the
    peer transport's wait; limit_ns 0 = 10 s). An expired wait sets the exchange status word (raised by
    ``check_status``)."""
    call("h3b_peer_wait", _p(flags), int(flags.numel()), int(epoch) & 0xFFFFFFFF, int(limit_ns), _stream(flags))


def selftest_wait_timeout(limit_ns: int, device: torch.device | str = "cuda") -> None:
    """Launches the bounded-wait self-test (a wait that nothing completes, given up after ``limit_ns``)."""
    call("h3b_selftest_wait_timeout", int(limit_ns), torch.cuda.current_stream(device).cuda_stream)


# ------------------------------------------------------------------------------------------------- VSA coarse step
def _i32_array(vals):
    import ctypes
    arr = (ctypes.c_int * max(1, len(vals)))(*[int(v) for v in vals])
    return arr


def qkv_prologue8(q, k, v, s1, tile_row0, vbs, wq, wk, cosb, sinb, inv_sq, inv_sk, qb, kb, vb, vs_blk, vs_head, qp,
                  kp, vp, heads, n_tiles, tile, eps, qc=None, kc=None, vc=None, qs_blk=None, ks_blk=None,
                  qk_int8: bool = False) -> None:
    """The reference op's argument order (h3fast.cu:889-927): RMSNorm + RoPE + tile means + E4M3 Q/K/V. 64-token
    tiles only; the compact dense-prefix copies (qc/kc/vc) are not supported. With qs_blk/ks_blk the Q/K scales are
    per (head, tile) instead of the static inv_sq/inv_sk; ``qk_int8`` (needs them) writes Q and K as symmetric int8
    (scale amax/127) for the attention's INT8 QK^T."""
    if tile != 64:
        raise RuntimeError("qkv_prologue8: 64-token tiles only")
    if qc is not None or kc is not None or vc is not None:
        raise RuntimeError("qkv_prologue8: the dense-prefix write-back (qc/kc/vc) is not supported")
    rows_pad = vb.shape[-2]
    n_ext = vs_blk.shape[-1]
    if vb.dtype == torch.float16:  # V as f16 (the decoded E4M3 values) for the f16-V attention
        if qs_blk is None or ks_blk is None:
            raise RuntimeError("qkv_prologue8: f16 V needs the per-tile Q/K scales")
        flags = 2 | (1 if qk_int8 else 0)
        call("h3b_qkv_prologue8_tiles", _p(q), _p(k), _p(v), q.stride(0), _p(s1), _p(tile_row0), _p(vbs), _p(wq),
             _p(wk), _p(cosb), _p(sinb), _p(qb), _p(kb), _p(vb), _p(qs_blk), _p(ks_blk), _p(vs_blk), _p(vs_head),
             _p(qp), _p(kp), _p(vp), int(heads), rows_pad, int(n_tiles), n_ext, float(eps), flags, _stream(q))
        return
    if qk_int8:
        call("h3b_qkv_prologue8_qk_int8", _p(q), _p(k), _p(v), q.stride(0), _p(s1), _p(tile_row0), _p(vbs), _p(wq),
             _p(wk), _p(cosb), _p(sinb), _p(qb), _p(kb), _p(vb), _p(qs_blk), _p(ks_blk), _p(vs_blk), _p(vs_head),
             _p(qp), _p(kp), _p(vp), int(heads), rows_pad, int(n_tiles), n_ext, float(eps), _stream(q))
        return
    call("h3b_qkv_prologue8", _p(q), _p(k), _p(v), q.stride(0), _p(s1), _p(tile_row0), _p(vbs), _p(wq), _p(wk),
         _p(cosb), _p(sinb), float(inv_sq), float(inv_sk), _p(qb), _p(kb), _p(vb), _p(qs_blk), _p(ks_blk), _p(vs_blk),
         _p(vs_head), _p(qp), _p(kp), _p(vp), int(heads), rows_pad, int(n_tiles), n_ext, float(eps), _stream(q))


def vsa_tile_quant(q, k, v, perm, tile_row0, vbs, qb, kb, vb, qs_blk, ks_blk, vs_blk, qp, kp, vp, n_tiles,
                   vs_head=None) -> None:
    """BASELINE config 4's prologue: head-major q/k/v [heads, S, 128] gathered into 64-token tiles through ``perm``,
    per-tile E4M3 Q/K/V, tile means; ``vs_head`` (zeroed by the caller) receives the per-head max V scale."""
    heads, seqlen = q.shape[-3], q.shape[-2]
    name = "h3b_vsa_tile_quant_v16" if vb.dtype == torch.float16 else "h3b_vsa_tile_quant"
    call(name, _p(q), _p(k), _p(v), heads, seqlen, _p(perm), _p(tile_row0), _p(vbs), _p(qb), _p(kb),
         _p(vb), _p(qs_blk), _p(ks_blk), _p(vs_blk), _p(vs_head), _p(qp), _p(kp), _p(vp), vb.shape[-2], int(n_tiles),
         vs_blk.shape[-1], _stream(q))


def head_tile_quant(x, s1, tile_row0, vbs, w, xb, xs_blk, xs_head, heads, n_tiles, eps=1e-6) -> None:
    """One tensor of the prologue's per-tile E4M3 form (cross-attention q, text k and v): optional row scale s1,
    optional per-head RMSNorm weight w, no RoPE. xb [heads, rows_pad, 128], xs_blk [heads, n_ext]."""
    name = "h3b_head_tile_quant_v16" if xb.dtype == torch.float16 else "h3b_head_tile_quant"
    call(name, _p(x), x.stride(0), _p(s1), _p(tile_row0), _p(vbs), _p(w), _p(xb), _p(xs_blk),
         _p(xs_head), int(heads), xb.shape[-2], int(n_tiles), xs_blk.shape[-1], float(eps), _stream(x))


def vsa_fp8(q8, k8, v8, q2k_idx, q2k_num, vbs, qk_coef, v_scale_blk, v_scale_head, lse=None, q_scale_blk=None,
            k_scale_blk=None, out=None):
    """FP8 block-sparse attention over the selected 64-key tiles, the reference op's arguments
    (h3fast.cu:860-862 / h3attn8.cu): returns ``out`` bf16 [1, heads, rows_pad, 128]. With q_scale_blk/k_scale_blk
    the Q/K scales are per tile and qk_coef is softmax scale * log2(e) only."""
    heads, rows_pad = q8.shape[-3], q8.shape[-2]
    n_ext = q2k_num.shape[-1]
    n = q2k_idx.shape[-1]
    if out is None:
        out = torch.zeros(1, heads, rows_pad, 128, device=q8.device, dtype=torch.bfloat16)
    if v8.dtype == torch.float16:  # V as f16 (the decoded E4M3 values): the same call on the f16-V kernel
        return vsa_fp8_ex(q8, k8, v8, out, q2k_idx, q2k_num, vbs, vbs, v_scale_blk, v_scale_head, qk_coef, heads,
                          n_ext, n, rows_pad, rows_pad, qs=q_scale_blk, ks=k_scale_blk, lse=lse, idx_ld=n,
                          q_scale_ld=n_ext, kv_scale_ld=n_ext)
    call("h3b_vsa_fp8", _p(q8), _p(k8), _p(v8), _p(q2k_idx), _p(q2k_num), _p(vbs), _p(q_scale_blk), _p(k_scale_blk),
         _p(v_scale_blk), _p(v_scale_head), float(qk_coef), _p(out), _p(lse), heads, n, n_ext, rows_pad, _stream(q8))
    return out


def vsa_status(reset: bool = False) -> int:
    import ctypes
    v = ctypes.c_int(0)
    call("h3b_vsa_status", ctypes.byref(v), int(reset))
    return int(v.value)


def tile_scores(qp: torch.Tensor, kp: torch.Tensor, sc: torch.Tensor, scale: float) -> None:
    heads, n = qp.shape[0], qp.shape[1]
    call("h3b_tile_scores", _p(qp), _p(kp), heads, n, float(scale), _p(sc), _stream(qp))


def topk_rows(scores, n, n_ext, prefix, starts, ends, ks, idx, num, split) -> None:
    """The reference op's arguments (h3fast.cu:929-957)."""
    heads = scores.numel() // (n * n)
    call("h3b_topk_rows", _p(scores), heads, int(n), int(n_ext), int(prefix), len(starts), _i32_array(starts),
         _i32_array(ends), _i32_array(ks), _p(idx), _p(num), int(bool(split)), _stream(scores))


def topk_pairs(scores, n, n_ext, prefix, starts, ends, ks, u_idx, u_mem, u_num, idx=None, num=None) -> None:
    """The reference op's arguments (h3fast.cu:959-987): per (head, pair of adjacent query tiles) the ascending union of
    both tiles' selections with membership bytes. ``idx``/``num``: optional topk_rows-shaped scratch."""
    heads = scores.numel() // (n * n)
    if idx is None:
        idx = torch.empty(heads, n_ext, n, device=scores.device, dtype=torch.int32)
    if num is None:
        num = torch.empty(heads, n_ext, device=scores.device, dtype=torch.int32)
    call("h3b_topk_pairs", _p(scores), heads, int(n), int(n_ext), int(prefix), len(starts), _i32_array(starts),
         _i32_array(ends), _i32_array(ks), _p(idx), _p(num), _p(u_idx), _p(u_mem), _p(u_num), _stream(scores))


def compressed_branch(sc: torch.Tensor, vp: torch.Tensor, oc: torch.Tensor) -> None:
    heads, n = vp.shape[0], vp.shape[1]
    call("h3b_compressed_branch", _p(sc), _p(vp), heads, n, _p(oc), _stream(sc))


def attn_gate_quant(ob, g, sg, oc, slot, n_tiles, tile, a, asf, sa, rows, o1=None, lse1a=None, lse1b=None,
                    lse2=None) -> None:
    """The reference op's arguments (h3fast.cu:1003-1029)."""
    W = ob.shape[-3] * ob.shape[-1]
    n1 = lse1a.shape[-1] if lse1a is not None else 0
    call("h3b_attn_gate_quant", _p(ob), _p(g), _p(sg), _p(oc), _p(slot), ob.shape[-2], int(n_tiles), int(tile),
         _p(a), _p(asf), _p(sa), int(rows), W, _p(o1), _p(lse1a), _p(lse1b), n1, _p(lse2), _stream(ob))


def vsa_pair(q8, k8, v8, u_idx, u_mem, u_num, vbs, qk_coef, v_scale_blk, v_scale_head, lse=None, q_scale_blk=None,
             k_scale_blk=None, out=None):
    """The pair form of the FP8 attention (vsa_pair_op, h3attn8.cu:44-77): per (head, pair of adjacent query tiles)
    the union list ``u_idx`` [heads * n_ext/2, max_u] of length ``u_num`` with membership bytes ``u_mem`` (bit 0:
    tile 2p, bit 1: tile 2p+1), as h3b_topk_pairs writes them. Q/K/V are the E4M3 [heads, rows_pad, 128] codes of
    vsa_fp8; returns ``out`` bf16 [1, heads, rows_pad, 128]."""
    heads, rows_pad = q8.shape[-3], q8.shape[-2]
    n_ext = rows_pad // 64
    if out is None:
        out = torch.zeros(1, heads, rows_pad, 128, device=q8.device, dtype=torch.bfloat16)
    if u_mem.dtype != torch.uint8 or u_mem.shape[-1] != u_idx.shape[-1]:
        raise RuntimeError("u_mem: uint8 with the shape of u_idx")
    return vsa_fp8_ex(q8, k8, v8, out, u_idx, u_num, vbs, vbs, v_scale_blk, v_scale_head, qk_coef, heads, n_ext,
                      vbs.numel(), rows_pad, rows_pad, qs=q_scale_blk, ks=k_scale_blk, lse=lse,
                      idx_ld=u_idx.shape[-1],
                      q_scale_ld=q_scale_blk.shape[-1] if q_scale_blk is not None else n_ext,
                      kv_scale_ld=v_scale_blk.shape[-1], _u_mem=u_mem)


def vsa_fp8_ex(q, k, v, out, idx, num, vbs_q, vbs_kv, vs, vs_head, qk_coef, heads, n_q_ext, n_kv, rows_chunk_q,
               rows_chunk_kv, chunks_q=1, chunks_kv=1, qs=None, ks=None, lse=None, idx_ld=None, q_scale_ld=None,
               kv_scale_ld=None, qk_int8: bool = False, _u_mem=None, shared_lists: bool = False, wide: bool = False):
    """General FP8 block-sparse attention (h3b_vsa_fp8_ex): chunked [chunks * heads, rows_chunk, 128] layouts (the
    all-to-all layout of sequence parallelism) and separate key/value tiles (cross-attention). ``shared_lists``: the
    list of each even query tile applies to it and the next tile (h3b_vsa_fp8_shared: one M=128 MMA stream per pair;
    cross-attention, dense layers). ``wide``: the wide-step kernel (h3b_vsa_fp8_ws: one weight-stationary M=64 MMA
    advances both key streams of a query tile per step; f16 V and E4M3 Q/K only)."""
    import ctypes

    from ._lib import VsaArgs
    x = VsaArgs()
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out), ("lse", lse), ("idx", idx), ("num", num),
                    ("vbs_q", vbs_q), ("vbs_kv", vbs_kv), ("qs", qs), ("ks", ks), ("vs", vs), ("vs_head", vs_head)):
        setattr(x, name, _p(t))
    x.qk_coef = float(qk_coef)
    x.heads, x.n_q_ext, x.n_kv = int(heads), int(n_q_ext), int(n_kv)
    x.idx_ld = int(idx_ld if idx_ld is not None else n_kv)
    x.q_scale_ld = int(q_scale_ld if q_scale_ld is not None else n_q_ext)
    x.kv_scale_ld = int(kv_scale_ld if kv_scale_ld is not None else n_kv)
    x.rows_chunk_q, x.rows_chunk_kv = int(rows_chunk_q), int(rows_chunk_kv)
    x.chunks_q, x.chunks_kv = int(chunks_q), int(chunks_kv)
    x.qk_int8 = int(bool(qk_int8))
    v16 = "_v16" if v.dtype == torch.float16 else ""  # f16 V (decoded E4M3 values) or E4M3 codes
    if wide:
        if not v16 or qk_int8 or shared_lists or _u_mem is not None:
            raise ValueError("the wide-step kernel takes f16 V, E4M3 Q/K and one key list per query tile")
        call("h3b_vsa_fp8_ws", ctypes.byref(x), _stream(q))
    elif _u_mem is not None:
        call("h3b_vsa_pair" + v16, ctypes.byref(x), _p(_u_mem), _stream(q))
    elif shared_lists:
        call("h3b_vsa_fp8_shared" + v16, ctypes.byref(x), _stream(q))
    else:
        call("h3b_vsa_fp8_ex" + v16, ctypes.byref(x), _stream(q))
    return out
