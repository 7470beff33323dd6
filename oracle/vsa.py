"""CPU restatement of the VSA path: prologue, tile scores, top-k selection, compressed branch, fine-step attention and
the attention-output gate -- TEST INFRASTRUCTURE ONLY.

Citations are to chronarion/fasth3-gb300. The tile scores and the selection are restated bit-exactly (fixed float32
order; integer selection). The prologue's E4M3 codes carry the same ambiguity window as ``oracle.quant`` (fast-math
reciprocals in the kernel); tile means are exact for power-of-two tile sizes (the kernel's reciprocal of the row count
is exact there). The fine step and the compressed branch are floating point and are compared within tolerance.
"""
from __future__ import annotations

import numpy as np

from . import quant as oq

D = 128
NWARP = 8


def order_key(f: np.ndarray) -> np.ndarray:
    """Order-preserving map of float32 bits to uint32 (h3fast.cu:519-522): -0.0 sorts below +0.0."""
    u = np.asarray(f, dtype=np.float32).view(np.uint32)
    return np.where(u >> 31, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_rows(scores: np.ndarray, n: int, n_ext: int, prefix: int, spans, split: bool):
    """topk_rows (h3fast.cu:524-588): per (head, query tile) the prefix tiles, then per span (start, end, k) the k
    largest keys with ties to the lowest column, ascending. Returns (idx [H, n_ext, n] with -1 past num, num)."""
    sc = np.asarray(scores, dtype=np.float32).reshape(-1, n)
    H = sc.shape[0] // n
    idx = np.full((H, n_ext, n), -1, dtype=np.int32)
    num = np.zeros((H, n_ext), dtype=np.int32)
    for row in range(H * n):
        h, q = divmod(row, n)
        if q < prefix:
            if not split:
                idx[h, q, :n] = np.arange(n)
            num[h, q] = 0 if split else n
            continue
        out = [] if split else list(range(prefix))
        for start, end, k in spans:
            length = end - start
            if k >= length:
                out.extend(range(start, end))
                continue
            keys = order_key(sc[row, start:end])
            # descending key, then ascending column
            order = np.lexsort((np.arange(length), -keys.astype(np.int64)))
            out.extend(sorted((start + order[:k]).tolist()))
        idx[h, q, :len(out)] = out
        num[h, q] = len(out)
    return idx, num


def topk_pairs(scores: np.ndarray, n: int, n_ext: int, prefix: int, spans):
    """topk_pairs (h3fast.cu:590-686): per (head, pair 2p, 2p+1 of query tiles) the ascending union of both tiles'
    topk_rows selections, with membership bits (1: tile 2p, 2: tile 2p+1); pad tiles (>= n) select nothing.
    Returns (u_idx [H * n_ext/2, n] with -1 past u_num, u_mem, u_num)."""
    idx, num = topk_rows(scores, n, n_ext, prefix, spans, False)
    H = idx.shape[0]
    P = n_ext // 2
    u_idx = np.full((H * P, n), -1, dtype=np.int32)
    u_mem = np.zeros((H * P, n), dtype=np.uint8)
    u_num = np.zeros(H * P, dtype=np.int32)
    for h in range(H):
        for p in range(P):
            mem = np.zeros(n, dtype=np.uint8)
            for t in range(2):
                r = 2 * p + t
                if r < n:
                    mem[idx[h, r, :num[h, r]]] |= np.uint8(1 << t)
            cols = np.nonzero(mem)[0]
            g = h * P + p
            u_idx[g, :cols.size] = cols
            u_mem[g, :cols.size] = mem[cols]
            u_num[g] = cols.size
    return u_idx, u_mem, u_num


def fma32(a, b, c) -> np.ndarray:
    """Correctly rounded float32 fused multiply-add, round_f32(a*b + c) with ties to even (IEEE 754 fusedMultiplyAdd),
    for float32 arrays. The product of two float32 values is exact in float64; TwoSum (Knuth) gives the float64 sum s and
    its exact error e (a*b + c = s + e). Rounding s to float32 gives the correctly rounded result except when s lies
    exactly halfway between two float32 neighbours (float64 rounding can land on a float32 midpoint, never cross one);
    there the sign of e decides."""
    a = np.asarray(a, dtype=np.float32).astype(np.float64)
    b = np.asarray(b, dtype=np.float32).astype(np.float64)
    c = np.asarray(c, dtype=np.float32).astype(np.float64)
    p = a * b
    s = p + c
    bb = s - p
    e = (p - (s - bb)) + (c - bb)
    t = s.astype(np.float32)
    td = t.astype(np.float64)
    d = s - td  # exact (Sterbenz)
    nb = np.nextafter(t, np.where(d > 0, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32))
    mid = (d != 0) & ((td + nb.astype(np.float64)) * 0.5 == s)
    fix = mid & (e != 0) & (np.sign(e) == np.sign(d))
    return np.where(fix, nb, t).astype(np.float32)


def tile_scores(qp: np.ndarray, kp: np.ndarray, scale: float) -> np.ndarray:
    """sc[h,i,j] = scale * sum_d qp[h,i,d] kp[h,j,d]: one float32 fused multiply-add per d, d ascending, then the scale
    multiply rounded to float32. The reference scores the tile means with torch.baddbmm (__init__.py:499-500, cuBLAS
    in TF32 by default or float32), whose internal order is not specified; this fixed order is the one the CUDA kernel
    implements, so scores and selection compare bit for bit."""
    qp = np.asarray(qp, dtype=np.float32)
    kp = np.asarray(kp, dtype=np.float32)
    acc = np.zeros((qp.shape[0], qp.shape[1], kp.shape[1]), dtype=np.float32)
    for d in range(qp.shape[2]):
        acc = fma32(qp[:, :, d, None], kp[:, None, :, d], acc)
    return (acc * np.float32(scale)).astype(np.float32)


def tile_means(x_rows: np.ndarray) -> np.ndarray:
    """Mean of a tile's rows [n, 128] in the kernel's order: warp w sums rows w, w+8, ... in order; warp sums are then
    added for w = 0..7; the total is multiplied by 1/n (h3fast.cu:358-373, 501-509)."""
    n = x_rows.shape[0]
    parts = np.zeros((NWARP, x_rows.shape[1]), dtype=np.float32)
    for i in range(n):
        parts[i % NWARP] = (parts[i % NWARP] + x_rows[i]).astype(np.float32)
    acc = np.zeros(x_rows.shape[1], dtype=np.float32)
    for w in range(NWARP):
        acc = (acc + parts[w]).astype(np.float32)
    return (acc * np.float32(np.float32(1.0) / np.float32(n))).astype(np.float32)


def _tile_codes(x_rows: np.ndarray):
    am = np.float32(np.abs(x_rows).max()) if x_rows.size else np.float32(0)
    s = np.float32(max(np.float32(am / oq.FP8_MAX), np.float32(1e-30)))
    u = (x_rows * np.float32(np.float32(1.0) / s)).astype(np.float32)
    return oq.e4m3_encode(u), s, oq._ambiguous(u, oq.e4m3_encode)


def vsa_tile_quant(q, k, v, perm, tile_row0, vbs, n_ext, tile=64):
    """BASELINE config 4's prologue: q/k/v [H, S, 128] (bf16 values) gathered into tiles through perm; per (head, tile)
    E4M3 codes with scale max(amax/448, 1e-30) for each of Q, K, V; tile means. Returns a dict."""
    H = q.shape[0]
    n_tiles = len(vbs)
    rows_pad = n_ext * tile
    out = {name: np.zeros((H, rows_pad, D), dtype=np.uint8) for name in ("qb", "kb", "vb")}
    out.update({name: np.zeros((H, rows_pad, D), dtype=bool) for name in ("qamb", "kamb", "vamb")})
    out.update({name: np.zeros((H, n_ext), dtype=np.float32) for name in ("qs", "ks", "vs")})
    out.update({name: np.zeros((H, n_tiles, D), dtype=np.float32) for name in ("qp", "kp", "vp")})
    perm = np.arange(int(np.sum(vbs))) if perm is None else np.asarray(perm)
    for h in range(H):
        for t in range(n_tiles):
            r0, n = int(tile_row0[t]), int(vbs[t])
            toks = perm[r0:r0 + n]
            for src, b, s, pname, amb in ((q, "qb", "qs", "qp", "qamb"), (k, "kb", "ks", "kp", "kamb"),
                                          (v, "vb", "vs", "vp", "vamb")):
                rows = np.asarray(src[h, toks], dtype=np.float32)
                codes, sc, am = _tile_codes(rows)
                out[b][h, t * tile:t * tile + n] = codes
                out[amb][h, t * tile:t * tile + n] = am
                out[s][h, t] = sc
                out[pname][h, t] = tile_means(rows)
    return out


def compressed_branch(sc: np.ndarray, vp: np.ndarray) -> np.ndarray:
    """softmax over key tiles of the scores, times the value tile means (fastvideo/models/dits/h3fast/__init__.py:509)."""
    s = np.asarray(sc, dtype=np.float64)
    p = np.exp(s - s.max(axis=-1, keepdims=True))
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("hij,hjd->hid", p, np.asarray(vp, dtype=np.float64)).astype(np.float32)


def vsa_fine(q, k, v, idx, num, vbs, sm_scale, tile=64):
    """Fine step of VSA: for every (head, query tile) exact softmax attention of its rows over the keys of its selected
    tiles (masked past vbs), float64. q/k/v: dequantized [H, rows_pad, 128]; idx/num as topk_rows. Returns
    [H, rows_pad, 128] float32 (rows past a tile's vbs and unselected tiles give 0)."""
    H, rows_pad, _ = q.shape
    out = np.zeros((H, rows_pad, D), dtype=np.float32)
    n_tiles = len(vbs)
    for h in range(H):
        for t in range(n_tiles):
            nq = int(vbs[t])
            cnt = int(num[h, t])
            if nq == 0 or cnt == 0:
                continue
            keys = np.concatenate([np.arange(b * tile, b * tile + int(vbs[b])) for b in idx[h, t, :cnt]])
            qq = np.asarray(q[h, t * tile:t * tile + nq], dtype=np.float64)
            s = qq @ np.asarray(k[h, keys], dtype=np.float64).T * sm_scale
            p = np.exp(s - s.max(axis=-1, keepdims=True))
            p /= p.sum(axis=-1, keepdims=True)
            out[h, t * tile:t * tile + nq] = (p @ np.asarray(v[h, keys], dtype=np.float64)).astype(np.float32)
    return out


def attn_gate_quant(ob, slot, rows, g=None, sg=None, oc=None, tile=64, fp4=False):
    """attn_gate_quant (h3fast.cu:688-741) without the merge: row r takes ob[h, slot[r]] for every head, adds
    oc[h, slot[r]//tile] * (sg[r] * g[r]) and is quantized like the row quantizers. ob [H, rows_pad, 128], g
    [rows, H*128], oc [H, n_tiles, 128]; all float32 holding bf16 values."""
    H = ob.shape[0]
    slot = np.asarray(slot, dtype=np.int64)
    o = np.transpose(np.asarray(ob, dtype=np.float32)[:, slot[:rows]], (1, 0, 2)).reshape(rows, H * D)
    if g is not None:
        cv = np.transpose(np.asarray(oc, dtype=np.float32)[:, slot[:rows] // tile], (1, 0, 2)).reshape(rows, H * D)
        sgg = (np.asarray(sg, dtype=np.float32)[:, None] * np.asarray(g, dtype=np.float32)).astype(np.float32)
        o = (o.astype(np.float64) + cv.astype(np.float64) * sgg.astype(np.float64)).astype(np.float32)
    if fp4:
        am = np.abs(o).max(axis=1).astype(np.float32)
        s = np.maximum((am / oq.FP4_RANGE).astype(np.float32), oq.FP4_MIN_SCALE).astype(np.float32)
        gs = (np.float32(1.0) / s).astype(np.float32)
        codes, bits, amb, sf_amb = oq.nvfp4_blocks(o, gs)
        return {"codes": codes, "sf_bits": bits, "s": s, "amb": amb, "sf_amb": sf_amb, "o": o}
    codes, s, amb = oq.fp8_rows_from_values(o)
    return {"codes": codes, "s": s, "amb": amb, "o": o}


def qkv_prologue8(q, k, v, s1, tile_row0, vbs, wq, wk, cosb, sinb, heads, s_q, s_k, eps=1e-5, n_ext=None, tile=64):
    """qkv_prologue8 (h3fast.cu:376-510) in float64 arithmetic rounded to bf16 where the kernel rounds: row scale s1,
    per-head RMSNorm with weights, rotate-half RoPE on the first 96 dims, bf16 q/k/v, E4M3 Q/K with static scales and
    V with one scale per (head, tile). The kernel's rsqrt and reciprocals are approximations, so compare the codes
    within one E4M3 step. Returns float values and codes."""
    rows = q.shape[0]
    n_tiles = len(vbs)
    n_ext = n_ext or n_tiles + n_tiles % 2
    rows_pad = n_ext * tile
    s = np.asarray(s1, dtype=np.float64)[:, None, None]
    qf = np.asarray(q, dtype=np.float64).reshape(rows, heads, D) * s
    kf = np.asarray(k, dtype=np.float64).reshape(rows, heads, D) * s
    vf = np.asarray(v, dtype=np.float64).reshape(rows, heads, D) * s

    def norm_rope(x, w):
        x = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * np.asarray(w, dtype=np.float64)
        c = np.asarray(cosb, dtype=np.float64)[:, None, :]
        sn = np.asarray(sinb, dtype=np.float64)[:, None, :]
        r, rest = x[..., :96], x[..., 96:]
        rot = np.concatenate([-r[..., 48:], r[..., :48]], -1)
        return np.concatenate([r * c + rot * sn, rest], -1)

    qo = oq.bf16_round(norm_rope(qf, wq).astype(np.float32))
    ko = oq.bf16_round(norm_rope(kf, wk).astype(np.float32))
    vo = oq.bf16_round(vf.astype(np.float32))
    out = {"q": qo, "k": ko, "v": vo}
    qb = np.zeros((heads, rows_pad, D), dtype=np.uint8)
    kb = np.zeros_like(qb)
    vb = np.zeros_like(qb)
    vs = np.ones((heads, n_ext), dtype=np.float32)
    for t in range(n_tiles):
        r0, n = int(tile_row0[t]), int(vbs[t])
        for h in range(heads):
            qb[h, t * tile:t * tile + n] = oq.e4m3_encode(qo[r0:r0 + n, h] / np.float32(s_q))
            kb[h, t * tile:t * tile + n] = oq.e4m3_encode(ko[r0:r0 + n, h] / np.float32(s_k))
            codes, sc, _ = _tile_codes(vo[r0:r0 + n, h])
            vb[h, t * tile:t * tile + n] = codes
            vs[h, t] = sc
    out.update(qb=qb, kb=kb, vb=vb, vs_blk=vs)
    return out
