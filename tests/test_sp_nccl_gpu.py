"""The sequence-parallel block loop on 2 GPUs: the output of two ranks (one process per GPU, head exchange around
attention over the peer transport -- copy engines into peer-mapped buffers, head groups pipelined; also with the tile
statistics sent by the SM put kernel -- and over NCCL all-to-alls) equals the single-GPU output bit for bit. Skipped
with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        cfg = pkg.model.DiTConfig(blocks=2)
        m = pkg.model.DiTModel.random(cfg, device=dev, seed=4)
        grid = (7, 16, 16)
        S = grid[0] * grid[1] * grid[2]
        g = torch.Generator(device=dev).manual_seed(8)
        x = torch.randn(1, S, cfg.hidden, device=dev, generator=g).bfloat16()
        ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
        temb = m.timestep_embedding(0.5)
        meta = pkg.runner.VsaMeta(grid=grid, topk=8)
        outs = {}
        for name in ("peer", "nccl", "peer+put"):
            exchange = name.split("+")[0]
            r = pkg.runner.H3FastRunner(m, pkg.sp.SeqParallel(), exchange=exchange)
            assert r.transport == exchange, (r.transport, r.transport_note)
            r.stats_put = name.endswith("+put")  # tile statistics by the SM kernel (h3b_peer_put)
            # two forwards: the peer transport's flags carry on counting from the first into the second
            outs[name] = [r.forward(x, temb, None, None, meta, context=ctx) for _ in range(2)]
            torch.cuda.synchronize()
            r.close()
        dist.barrier()
        ref = pkg.runner.H3FastRunner(m).forward(x, temb, None, None, meta, context=ctx)
        torch.cuda.synchronize()
        bad = [f"{ex} forward {k}: {int((o != ref).sum())} elements differ" for ex, os_ in outs.items()
               for k, o in enumerate(os_) if not torch.equal(o.view(torch.int16), ref.view(torch.int16))]
        q.put((rank, "ok" if not bad else "mismatch: " + "; ".join(bad)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_nccl_block_loop_equals_single_gpu(h3b):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res == {0: "ok", 1: "ok"}, res
