"""Sequence-parallel host logic on CPU ranks (gloo, world size 2): the head all-to-all layouts, tile sharding, and
failure detection (a rank that dies before an exchange makes its peer's collective fail instead of hang)."""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path.insert(0, str(ROOT))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        import __graft_entry__  # noqa: F401
        pkg = __graft_entry__.load_package()
        if ":" in fn_name:  # a rank body of another test module, "module:function"
            import importlib
            mod, fn = fn_name.split(":")
            getattr(importlib.import_module(mod), fn)(rank, world, pkg)
        else:
            globals()[fn_name](rank, world, pkg)
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(fn_name, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, msg = q.get(timeout=timeout)
        results[rank] = msg
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


# ------------------------------------------------------------------------------------------------ rank bodies
def body_exchange(rank, world, pkg):
    from fasth3_b200.sp import SeqParallel
    sp = SeqParallel()
    H, R, D = 4, 6, 3
    full = torch.arange(H * world * R * D, dtype=torch.float32).view(H, world * R, D)  # [H, all rows, D]
    mine = full[:, rank * R:(rank + 1) * R].contiguous()
    got = sp.seq_to_heads(mine)  # [P, Hl, R, D]
    h0, h1 = sp.heads(H)
    for p in range(world):
        assert torch.equal(got[p], full[h0:h1, p * R:(p + 1) * R]), p
    back = sp.heads_to_seq(got)
    assert torch.equal(back, mine)
    stats = full[:, rank * R:(rank + 1) * R, 0].contiguous()  # [H, n_local]
    merged = sp.tile_stats_to_heads(stats)
    assert torch.equal(merged, full[h0:h1, :, 0])


def body_layout(rank, world, pkg):
    from fasth3_b200.layout import tile_layout
    from fasth3_b200.sp import SeqParallel
    sp = SeqParallel()
    lay = tile_layout(7, 12, 20, pad_to=2 * world)  # last time slab has 3 frames: 48-token tiles
    first, last = sp.tiles(lay.n_ext)
    part = lay.shard(first, last)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([part.rows]))
    m = int(max(int(s) for s in sizes))
    padded = torch.full((m,), -1, dtype=torch.int64)
    padded[:part.rows] = part.perm
    perms = [torch.zeros(m, dtype=torch.int64) for _ in sizes]
    dist.all_gather(perms, padded)  # gloo gathers equal sizes only
    assert torch.equal(torch.cat([p[:int(s)] for p, s in zip(perms, sizes)]), lay.perm)
    assert (part.vbs <= 64).all() and part.rows == int(part.vbs.sum())


def body_runner_exchange(rank, world, pkg):
    """The runner's exchange object over real ranks: the all-to-all layouts and the final gather with unequal rows."""
    from fasth3_b200.runner import _Exchange
    from fasth3_b200.sp import SeqParallel
    ex = _Exchange(SeqParallel())
    H, R, D = 4, 6, 3
    full = torch.arange(H * world * R * D, dtype=torch.float32).view(H, world * R, D)
    mine = full[:, rank * R:(rank + 1) * R].contiguous()
    got = torch.empty(world, H // world, R, D)
    ex.seq_to_heads([mine], [got])
    back = torch.empty_like(mine)
    ex.heads_to_seq([got], [back])
    assert torch.equal(back, mine)
    rows = [5 + p for p in range(world)]  # unequal row counts per rank
    x = torch.full((rows[rank], 2), float(rank))
    out = ex.all_gather_rows([x], rows)
    assert torch.equal(out, torch.cat([torch.full((r, 2), float(p)) for p, r in enumerate(rows)]))


def body_peer_dies(rank, world, pkg):
    from fasth3_b200.sp import SeqParallel
    sp = SeqParallel()
    if rank == 1:
        raise RuntimeError("injected failure before the exchange")
    x = torch.zeros(4, 2, 2)
    sp.seq_to_heads(x)  # must raise (peer gone / timeout), not hang


# ------------------------------------------------------------------------------------------------ tests
def test_head_all_to_all_layouts():
    res = _run("body_exchange")
    assert all(v == "ok" for v in res.values()), res


def test_tile_sharding_covers_the_latent():
    res = _run("body_layout")
    assert all(v == "ok" for v in res.values()), res


def test_runner_exchange_over_real_ranks():
    res = _run("body_runner_exchange")
    assert all(v == "ok" for v in res.values()), res


def test_dead_peer_fails_the_exchange_instead_of_hanging():
    res = _run("body_peer_dies", timeout=90)
    assert res[1].startswith("error: RuntimeError: injected failure"), res[1]
    assert res[0].startswith("error:"), res[0]  # the survivor's collective errored out


def test_layout_single_process_properties():
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from fasth3_b200.layout import rope_3d, tile_layout
    lay = tile_layout(31, 48, 84, pad_to=16)  # 124,992 tokens
    assert lay.rows == 124992 and lay.n_tiles == 2016 and lay.n_ext == 2016
    assert int(lay.vbs.min()) == 48 and int(lay.vbs.max()) == 64
    assert sorted(lay.perm.tolist()) == list(range(lay.rows))
    cos, sin = rope_3d(lay)
    assert cos.shape == (lay.rows, 96) and sin.shape == (lay.rows, 96)
    with pytest.raises(ValueError):
        from fasth3_b200.sp import SeqParallel
        SeqParallel().tiles(2015)
