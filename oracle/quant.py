"""CPU restatement of the activation quantizers and weight packing -- TEST INFRASTRUCTURE ONLY.

Every float32 operation is rounded where the reference kernel rounds it. The reference kernel is built with
``--use_fast_math`` (fastvideo/models/dits/h3fast/__init__.py:42): its reciprocal ``1.f/s``, the divisions ``gs/sf``
and ``ss/C`` and ``rsqrtf`` are hardware approximations within a few ulp of the IEEE results this file computes. So each
quantizer also returns an *ambiguity mask*: the codes whose pre-rounding value lies within a relative ``DELTA`` of a
rounding boundary, where those few ulp can legitimately flip the code. Outside the mask the oracle is exact; the GPU is
held bit-exact to the reference kernel itself on the GPU.
"""
from __future__ import annotations

import numpy as np
import torch

FP8_MAX = np.float32(448.0)
FP8_MIN_SCALE = np.float32(1.0 / (448.0 * 512.0))  # h3fast.cu:23 kMinScale; FastVideo's FP8_MIN_SCALE (not vendored)
FP4_RANGE = np.float32(448.0 * 6.0)                 # h3fast.cu:24
FP4_MIN_SCALE = np.float32(1e-12)                   # h3fast.cu:25
SIXTH = np.float32(1.0 / 6.0)
DELTA = 1e-6  # relative window around rounding boundaries (~17 float32 ulp; the approximations are <= 4 ulp)

f32 = np.float32


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even) -> float32."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Saturating round-to-nearest-even float32 -> e4m3 bytes (cvt.rn.satfinite semantics for finite inputs)."""
    x = np.clip(np.asarray(x, dtype=np.float32), -FP8_MAX, FP8_MAX)
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint8)).view(torch.float8_e4m3fn).float().numpy()


E2M1_VALUES = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)


def e2m1_encode(x: np.ndarray) -> np.ndarray:
    """Saturating round-to-nearest-even float32 -> e2m1 nibble codes 0..15 (bit 3 = sign, kept for -0)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x)
    # magnitude code: ties go to the even code (0, 1.0, 2.0, 4.0 have even mantissa)
    mag = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return mag | (np.signbit(x).astype(np.uint8) << 3)


def e2m1_decode(c: np.ndarray) -> np.ndarray:
    return E2M1_VALUES[np.asarray(c, dtype=np.int64)]


def sf_atom_offset(row, col, sf_cols):
    """h3fast.cu:94-97 layout_128x4 byte offset (vectorised)."""
    row = np.asarray(row, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    return ((row >> 7) * (sf_cols >> 2) * 512 + (col >> 2) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4
            + (col & 3))


def _ambiguous(u: np.ndarray, encode, mag: np.ndarray | None = None) -> np.ndarray:
    """Codes that a relative error of DELTA could flip. ``mag`` (same shape as u, in u's units) is the magnitude the
    error is relative to when u comes out of a cancellation (x * (1 + scale) + shift near zero): the window is then
    DELTA * (|u| + mag) instead of DELTA * |u|."""
    u = np.asarray(u, dtype=np.float64)
    err = np.abs(u) * DELTA if mag is None else (np.abs(u) + np.abs(np.asarray(mag, dtype=np.float64))) * DELTA
    lo = encode((u - err).astype(np.float32))
    hi = encode((u + err).astype(np.float32))
    return lo != hi


def butterfly_sum(a: np.ndarray) -> np.ndarray:
    """The xor-shuffle all-reduce over the last axis (32 lanes): lane l adds lane l^16, then l^8, ... (h3fast.cu:
    142-147). Pairwise halving reproduces its float32 tree exactly."""
    a = a.astype(np.float32)
    while a.shape[-1] > 1:
        h = a.shape[-1] // 2
        a = (a[..., :h] + a[..., h:]).astype(np.float32)
    return a[..., 0]


def block_sum(v: np.ndarray, serial: bool = True) -> np.ndarray:
    """Row sum of ``v`` [rows, C] in the reference's order: thread t owns elements [8t, 8t+8) summed left to right,
    a butterfly per warp, warp partials (zero past the last warp) butterflied again (h3fast.cu:139-152)."""
    rows, C = v.shape
    T = C // 8
    NW = T // 32
    t = v.reshape(rows, T, 8).astype(np.float32)
    acc = np.zeros((rows, T), dtype=np.float32)
    for i in range(8):
        acc = (acc + t[:, :, i]).astype(np.float32)
    warp = butterfly_sum(acc.reshape(rows, NW, 32))
    stage = np.zeros((rows, 32), dtype=np.float32)
    stage[:, :NW] = warp
    return butterfly_sum(stage)


def block_sum_sq(v: np.ndarray) -> np.ndarray:
    """As block_sum but accumulating v*v with a fused multiply-add per element (the GPU contracts ``ss += v*v``)."""
    rows, C = v.shape
    T = C // 8
    NW = T // 32
    t = v.reshape(rows, T, 8).astype(np.float64)
    acc = np.zeros((rows, T), dtype=np.float32)
    for i in range(8):
        acc = (acc.astype(np.float64) + t[:, :, i] * t[:, :, i]).astype(np.float32)
    warp = butterfly_sum(acc.reshape(rows, NW, 32))
    stage = np.zeros((rows, 32), dtype=np.float32)
    stage[:, :NW] = warp
    return butterfly_sum(stage)


def ln_row_shape(C: int) -> tuple[int, int]:
    """(K, G) of the LayerNorm row layout (fasth3-gb300_b200/csrc/quant.cu, LnRowShape): G threads per row, thread t
    owning the 8-element chunks t, t + G, ..., t + (K - 1) G; K the largest of 5, 4, 3, 2 giving whole warps, else 1."""
    chunks = C // 8
    for k in (5, 4, 3, 2):
        if chunks % k == 0 and (chunks // k) % 32 == 0:
            return k, chunks // k
    return 1, chunks


def ln_row_sum(v: np.ndarray, squares: bool = False) -> np.ndarray:
    """Row sum in the LayerNorm quantizer's order (fasth3-gb300_b200/csrc/quant.cu, ln_thread_sum and the kernels'
    reductions): each thread of the row layout (ln_row_shape) keeps two float32 accumulators, one for the even and one
    for the odd elements of its chunks, advanced chunk by chunk (``squares``: v*v added with one fused multiply-add per
    element); the thread's sum is the two accumulators added, each warp butterflies its 32 thread sums, and the warp
    sums are added in warp order."""
    rows, C = v.shape
    K, G = ln_row_shape(C)
    t = np.asarray(v, dtype=np.float32).reshape(rows, K, G, 4, 2)  # [row, k, thread, pair, even/odd]
    acc = np.zeros((rows, G, 2), dtype=np.float32)
    for k in range(K):
        for p in range(4):
            x = t[:, k, :, p, :]
            if squares:
                x64 = x.astype(np.float64)
                acc = (acc.astype(np.float64) + x64 * x64).astype(np.float32)
            else:
                acc = (acc + x).astype(np.float32)
    th = (acc[..., 0] + acc[..., 1]).astype(np.float32)
    warp = butterfly_sum(th.reshape(rows, G // 32, 32))
    tot = warp[:, 0]
    for q in range(1, G // 32):
        tot = (tot + warp[:, q]).astype(np.float32)
    return tot


def fp8_rows_from_values(v: np.ndarray, mag: np.ndarray | None = None):
    """FP8 row quantization of float32 rows (h3fast.cu:256-262): returns (codes, scale, ambiguity). ``mag``: the
    pre-cancellation magnitude of v for the ambiguity window (see _ambiguous)."""
    am = np.abs(v).max(axis=1).astype(np.float32)
    s = np.maximum((am / FP8_MAX).astype(np.float32), FP8_MIN_SCALE).astype(np.float32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    u = (v * inv[:, None]).astype(np.float32)
    m = None if mag is None else np.abs(mag) * inv[:, None]
    return e4m3_encode(u), s, _ambiguous(u, e4m3_encode, m)


def nvfp4_blocks(v: np.ndarray, gs: np.ndarray, mag: np.ndarray | None = None):
    """NVFP4 block math of h3fast.cu:99-119 for rows ``v`` [rows, K] with global factor ``gs`` [rows] (row mode) or
    scalar (tensor mode). Returns (codes [rows, K] 0..15, sf bytes [rows, K/16], nibble ambiguity, sf ambiguity).
    ``mag``: the pre-cancellation magnitude of v for the ambiguity window (see _ambiguous)."""
    rows, K = v.shape
    gs = np.broadcast_to(np.asarray(gs, dtype=np.float32).reshape(-1, 1), (rows, 1)).astype(np.float32)
    blk = v.reshape(rows, K // 16, 16).astype(np.float32)
    vmax = np.abs(blk).max(axis=2).astype(np.float32)
    x = (gs * (vmax * SIXTH).astype(np.float32)).astype(np.float32)
    bits = e4m3_encode(x)
    sf_amb = _ambiguous(x, e4m3_encode)
    sf = e4m3_decode(bits)
    with np.errstate(divide="ignore", invalid="ignore"):
        m = np.where((vmax != 0) & (sf != 0), (gs / sf).astype(np.float32), np.float32(0)).astype(np.float32)
    u = (blk * m[:, :, None]).astype(np.float32)
    codes = e2m1_encode(u)
    mu = None if mag is None else np.abs(np.asarray(mag, dtype=np.float32).reshape(rows, K // 16, 16)) * m[:, :, None]
    amb = _ambiguous(u, e2m1_encode, mu) | sf_amb[:, :, None]
    return codes.reshape(rows, K), bits, amb.reshape(rows, K), sf_amb


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[rows, K] codes -> [rows, K/2] bytes, element 2i in the low nibble (h3fast.cu:80-83)."""
    c = codes.astype(np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q, dtype=np.uint8)
    out = np.empty((q.shape[0], q.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = q & 15
    out[:, 1::2] = q >> 4
    return out


def swizzle_sf(bits: np.ndarray) -> np.ndarray:
    """[rows, K/16] scale bytes -> the flat 128x4-atom buffer [pad128(rows), K/16] (zeros in the padding)."""
    rows, cols = bits.shape
    pad = (rows + 127) // 128 * 128
    out = np.zeros(pad * cols, dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    out[sf_atom_offset(r, c, cols)] = bits
    return out.reshape(pad, cols)


def unswizzle_sf(buf: np.ndarray, rows: int, cols: int) -> np.ndarray:
    flat = np.asarray(buf, dtype=np.uint8).reshape(-1)
    r, c = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    return flat[sf_atom_offset(r, c, cols)]


# ----------------------------------------------------------------------------------------------- the row kernel
def resid_norm_quant(x, y=None, sy=None, gate=None, idx=None, nw=None, shift=None, scale=None, eps=1e-5,
                     norm="rms", fp4=False):
    """Restatement of resid_norm_quant (h3fast.cu:188-265) plus the LayerNorm variant BASELINE config 3 names.

    Inputs are float32 arrays holding bf16 values: x, y [rows, C]; sy [rows]; gate/shift/scale tables [T, C];
    idx [rows] int; nw [C]. Returns a dict with xo (float32 bf16 values), and with a norm: h (FP8 codes [rows, C] or
    packed NVFP4 [rows, C/2]), hs [rows], hsf (swizzled, NVFP4), amb (ambiguity mask over h's codes), sf_amb.
    """
    v = np.asarray(x, dtype=np.float32)
    rows, C = v.shape
    idx = np.zeros(rows, dtype=np.int64) if idx is None else np.asarray(idx, dtype=np.int64)
    out = {}
    if y is not None:
        g = np.asarray(gate, dtype=np.float32)[idx]
        b = (np.asarray(sy, dtype=np.float32)[:, None] * np.asarray(y, dtype=np.float32)).astype(np.float32)
        # x + g * (s * b): the product-add contracts to one fma on the GPU; bf16 rounding makes it immaterial
        # except at bf16 ties, which the float64 evaluation below resolves the same way as the fma.
        v = bf16_round((v.astype(np.float64) + g.astype(np.float64) * b.astype(np.float64)).astype(np.float32))
        out["xo"] = v
    if norm in (None, "none"):
        return out
    sc = np.asarray(scale, dtype=np.float32)[idx]
    sf = np.asarray(shift, dtype=np.float32)[idx]
    one_sc = (np.float32(1.0) + sc).astype(np.float32)
    if norm == "rms":
        ss = block_sum_sq(v)
        t = ((ss / np.float32(C)).astype(np.float32) + np.float32(eps)).astype(np.float32)
        rs = (1.0 / np.sqrt(t.astype(np.float64))).astype(np.float32)
        w = np.asarray(nw, dtype=np.float32)
        p = ((v * rs[:, None]).astype(np.float32) * w[None, :]).astype(np.float32)
        m = (p.astype(np.float64) * one_sc + sf).astype(np.float32)
    elif norm == "layer":  # the LayerNorm variant's own summation order (ln_row_sum)
        mean = (ln_row_sum(v) / np.float32(C)).astype(np.float32)
        d = (v - mean[:, None]).astype(np.float32)
        var = (ln_row_sum(d, squares=True) / np.float32(C)).astype(np.float32)
        rs = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float64))).astype(np.float32)
        p = (d * rs[:, None]).astype(np.float32)
        m = (p.astype(np.float64) * one_sc + sf).astype(np.float32)
    else:
        raise ValueError(norm)
    out["m"] = m
    mag = np.abs(p.astype(np.float64) * one_sc).astype(np.float32)  # the shift can cancel the normalized term
    if fp4:
        am = np.abs(m).max(axis=1).astype(np.float32)
        s = np.maximum((am / FP4_RANGE).astype(np.float32), FP4_MIN_SCALE).astype(np.float32)
        gs = (np.float32(1.0) / s).astype(np.float32)
        codes, bits, amb, sf_amb = nvfp4_blocks(m, gs, mag)
        out.update(h=pack_nibbles(codes), codes=codes, hs=s, hsf=swizzle_sf(bits), sf_bits=bits, amb=amb,
                   sf_amb=sf_amb)
    else:
        codes, s, amb = fp8_rows_from_values(m, mag)
        out.update(h=codes, hs=s, amb=amb)
    return out


def quant_fp8_rows(x):
    """Per-token FP8 of bf16-valued float32 rows (BASELINE config 1's activation quantizer)."""
    codes, s, amb = fp8_rows_from_values(np.asarray(x, dtype=np.float32))
    return codes, s, amb


def quant_nvfp4_tensor(x):
    """Per-tensor NVFP4: s = max(amax/2688, 1e-12), gs = 1/s, block math of h3fast.cu:99-119.
    Returns (packed [rows, K/2], swizzled sf [pad128(rows), K/16], s, nibble ambiguity, sf ambiguity [rows, K/16])."""
    v = np.asarray(x, dtype=np.float32)
    am = np.float32(np.abs(v).max()) if v.size else np.float32(0)
    s = np.maximum(np.float32(am / FP4_RANGE), FP4_MIN_SCALE).astype(np.float32)
    gs = np.float32(np.float32(1.0) / s)
    codes, bits, amb, sf_amb = nvfp4_blocks(v, gs)
    return pack_nibbles(codes), swizzle_sf(bits), s, amb, sf_amb


def dequant_nvfp4(q: np.ndarray, sf_buf: np.ndarray, rows: int, K: int, s) -> np.ndarray:
    """Codes x block scale x global (row or tensor) scale -> float32 [rows, K] (h3fast.cu:758-779)."""
    vals = e2m1_decode(unpack_nibbles(q)[:rows]).reshape(rows, K // 16, 16)
    sfv = e4m3_decode(unswizzle_sf(sf_buf, rows, K // 16))
    s = np.asarray(s, dtype=np.float32).reshape(-1, 1, 1) if np.ndim(s) else np.float32(s)
    return (vals * sfv[:, :, None] * s).reshape(rows, K).astype(np.float32)


def quantize_fp8_weight(weight: torch.Tensor, granularity: str = "tensor") -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 weight quantization (patches/fastvideo-a01c50a.patch:384-394) on the CPU in torch: the scale is taken in
    float32, rounded to the weight dtype before dividing, the quotient clamped to +-448 and cast to e4m3."""
    w = weight.detach()
    if granularity == "channel":
        amax = w.abs().amax(dim=1).nan_to_num().float()
        scale = (amax / float(FP8_MAX)).clamp(min=float(FP8_MIN_SCALE))
        divisor = scale.to(w.dtype).unsqueeze(1)
    else:
        amax = w.abs().amax().nan_to_num().float()
        scale = (amax / float(FP8_MAX)).clamp(min=float(FP8_MIN_SCALE)).view(1)
        divisor = scale.to(w.dtype)
    q = (w / divisor).clamp(-float(FP8_MAX), float(FP8_MAX)).to(torch.float8_e4m3fn)
    return q.contiguous(), scale.float()
