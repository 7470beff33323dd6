"""The peer transport's host logic on CPU: the byte geometry of every copy of the head exchange (against the
all-to-all layouts the NCCL and emulated transports produce), and a failure on one rank while the peer arena is set
up reaching every rank as an error instead of a hang (gloo ranks, the C calls replaced by a fake)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_sp_gloo import _run


def _copy2d(dst: np.ndarray, doff: int, dpitch: int, src: np.ndarray, soff: int, spitch: int, w: int, h: int):
    """cudaMemcpy2D on byte arrays."""
    for row in range(h):
        dst[doff + row * dpitch:doff + row * dpitch + w] = src[soff + row * spitch:soff + row * spitch + w]


def _bytes(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).reshape(-1).numpy().copy()


@pytest.mark.parametrize("P,H,G,planes,es", [(2, 8, 2, 3, 1), (2, 8, 4, 2, 1), (4, 8, 2, 1, 2), (8, 40, 5, 3, 1),
                                             (2, 40, 4, 3, 1)])
def test_qkv_and_out_geometry_match_the_all_to_all(h3b, P, H, G, planes, es):
    from fasth3_b200.runner import VirtualSeqParallel, _Exchange
    from fasth3_b200.sp import peer_copy_plan
    R, D = 4, 2  # rows per rank, head width (small: only the geometry is checked)
    Hl, Hg = H // P, H // P // G
    dt = torch.uint8 if es == 1 else torch.float16
    gen = torch.Generator().manual_seed(P * 100 + H + G)
    src = [torch.randint(0, 250, (planes, H, R, D), generator=gen).to(dt) for _ in range(P)]
    # what the emulated transport delivers, plane by plane: [G, P, Hg, R, D] per rank
    ex = _Exchange(VirtualSeqParallel(P))
    want = [torch.zeros(planes, G, P, Hg, R, D, dtype=dt) for _ in range(P)]
    for j in range(planes):
        ex.heads_exchange([s[j] for s in src], [w[j] for w in want])
    dims = {"P": P, "H": H, "G": G, "R": R, "D": D, "es": es, "planes": planes}
    got = [np.zeros(want[0].numel() * es, dtype=np.uint8) for _ in range(P)]
    for r in range(P):
        sb = _bytes(src[r])
        for p in range(P):
            for g in range(G):
                so, sp, do, dp, w, h = peer_copy_plan("qkv", r, p, g, dims)
                _copy2d(got[p], do, dp, sb, so, sp, w, h)
    for p in range(P):
        assert np.array_equal(got[p], _bytes(want[p])), p
    # and back: attention outputs [G, P, Hg, R, D] -> [H, R, D]
    outs = [torch.randn(G, P, Hg, R, D, generator=gen).to(torch.bfloat16) for _ in range(P)]
    back = [torch.zeros(H, R, D, dtype=torch.bfloat16) for _ in range(P)]
    ex.heads_return(outs, back)
    dims["es"] = 2
    got = [np.zeros(H * R * D * 2, dtype=np.uint8) for _ in range(P)]
    for r in range(P):
        sb = _bytes(outs[r])
        for p in range(P):
            for g in range(G):
                so, sp, do, dp, w, h = peer_copy_plan("out", r, p, g, dims)
                _copy2d(got[p], do, dp, sb, so, sp, w, h)
    for p in range(P):
        assert np.array_equal(got[p], _bytes(back[p])), p


@pytest.mark.parametrize("P,H,n,T", [(2, 8, 3, 1), (4, 8, 2, 5), (8, 40, 4, 1), (8, 40, 2, 3)])
def test_tile_statistics_land_in_global_tile_order(h3b, P, H, n, T):
    from fasth3_b200.sp import peer_copy_plan
    Hl = H // P
    full = torch.arange(H * P * n * T, dtype=torch.float32).view(H, P * n, T)  # [H, all tiles, T]
    dims = {"P": P, "H": H, "G": 1, "R": 64, "D": 128, "es": 4, "n": n, "T": T}
    for p in range(P):  # receiver p: its heads, every tile
        got = np.zeros(Hl * P * n * T * 4, dtype=np.uint8)
        for r in range(P):  # sender r: every head of its tiles
            sb = _bytes(full[:, r * n:(r + 1) * n])
            so, sp, do, dp, w, h = peer_copy_plan("stats", r, p, 0, dims)
            _copy2d(got, do, dp, sb, so, sp, w, h)
        assert np.array_equal(got, _bytes(full[p * Hl:(p + 1) * Hl])), p


# ------------------------------------------------------------------------------------------------ arena set-up
def body_arena_alloc_fails_on_one_rank(rank, world, pkg):
    """Rank 1's allocation fails; rank 0's succeeds. Both ranks must raise (after the same collectives) and rank 0
    must free what it allocated."""
    import fasth3_b200._lib as lib
    from fasth3_b200.sp import PeerArena, SeqParallel
    calls = []

    def fake_call(name, *args):
        calls.append(name)
        if name == "h3b_peer_alloc":
            if rank == 1:
                raise RuntimeError("h3b_peer_alloc: injected failure")
            args[2]._obj.value = 0x10000  # the out-pointer (ctypes.byref) gets a fake device address
        elif name == "h3b_peer_open":
            raise AssertionError("no rank may open a peer when one rank has no arena")

    lib.call = fake_call
    try:
        PeerArena(SeqParallel(), "cuda:0", {"x": ((64,), torch.uint8)}, 3)
    except RuntimeError as exc:
        assert "rank 1" in str(exc) and "injected failure" in str(exc), exc
        if rank == 0:
            assert calls == ["h3b_peer_alloc", "h3b_peer_export", "h3b_peer_free"], calls
        return
    raise AssertionError("the arena was set up although rank 1 failed")


def test_arena_setup_failure_reaches_every_rank():
    res = _run("test_peer_plan:body_arena_alloc_fails_on_one_rank")
    assert all(v == "ok" for v in res.values()), res


# ------------------------------------------------------------------------------------------------ SM statistics put
class _FakeArena:
    """Addresses only: rank p's allocation at (p + 1) << 40, region k of ``names`` at k << 32, flags at 1 << 39."""

    def __init__(self, names, world):
        self.names, self.world = list(names), world

    def ptr(self, p, name, off=0):
        return ((p + 1) << 40) + (self.names.index(name) << 32) + off

    def flag(self, p, slot, sender):
        return ((p + 1) << 40) + (1 << 39) + 4 * (slot * self.world + sender)


_S5, _S6 = ("qs", "ks", "vs", "qp", "kp"), ("qs", "ks", "vs", "qp", "kp", "vp")


@pytest.mark.parametrize("P,r,stats", [(8, 3, _S5), (2, 1, _S6), (11, 0, _S6)])
def test_stats_put_arguments_follow_the_copy_plan(h3b, P, r, stats):
    """The tile statistics' h3b_peer_put arguments (runner.stats_put): one copy per (receiver, statistic) with the
    geometry the copy-engine path uses, each receiver's flag slot 0 for this sender, built once per layout; when
    the copies exceed one put (64) the runner keeps the copy-engine path."""
    import types

    from fasth3_b200._lib import PEER_PUT_MAX_COPIES
    from fasth3_b200.runner import H3FastRunner
    H, n, D = 8 * P, 6, 128
    b = {nm: torch.zeros(H, n, *((D,) if nm.endswith("p") else ()), dtype=torch.float32) for nm in stats}
    st = types.SimpleNamespace(b=b, n_local=n, rows_pad=n * 64, arena=_FakeArena([nm + "_all" for nm in stats], P))
    me = types.SimpleNamespace(ex=types.SimpleNamespace(world=P, sp=types.SimpleNamespace(rank=r)), dev="cpu",
                               heads=H, head_groups=1, head_dim=D)
    me._peer_dims = types.MethodType(H3FastRunner._peer_dims, me)
    me._stats_plan = types.MethodType(H3FastRunner._stats_plan, me)
    put = H3FastRunner._peer_stats_put(me, st, stats)
    if P * len(stats) > PEER_PUT_MAX_COPIES:
        assert put is None
        return
    arr, count, flags, n_flags, counter = put
    assert count == P * len(stats) and n_flags == P and int(counter) == 0
    for p in range(P):
        assert flags[p] == st.arena.flag(p, 0, r)
        for j, nm in enumerate(stats):
            c = arr[p * len(stats) + j]
            so, sp_, do, dp, w, rows = me._stats_plan(st, nm, p)
            want = (st.arena.ptr(p, nm + "_all", do), b[nm].data_ptr() + so, dp, sp_, w, rows)
            assert (c.dst, c.src, c.dpitch, c.spitch, c.width, c.height) == want, (p, nm)
    assert H3FastRunner._peer_stats_put(me, st, stats) is put  # cached per layout
