"""Benchmark of the B200 quantized DiT-linear hot path (BASELINE.json metric "NVFP4/FP8 DiT-linear TFLOPS").

Workload (the configuration the metric is quoted on): one NVFP4 DiT linear per step --
X bf16 [32768 x 5120] (N(0,1), 0.5% of columns x30) -> per-tensor NVFP4 quantization (amax pass + e2m1/ue4m3 pack)
-> block-scaled tcgen05 GEMM with the pre-packed weight W [13824 x 5120] -> Y bf16 [32768 x 13824].
2*M*N*K = 4.638 TFLOP per step. Inputs (X 335 MB) and outputs (Y 906 MB) are larger than the 126 MB L2, so no flush.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; each rank processes its own 32768-token shard (weak scaling, no data
collective: the linear is row-independent). Rank 0 prints one JSON line.
Secondary lines beside the headline: the FP8 linear and block chain (config 3), the VSA step (config 4), offline
weight packing, and the 50-block DiT step (config 5), on one GPU also with token reduction over blocks 4..29 and with
INT8 QK^T (``--no-dit-extras`` skips those two).
``--impl reference`` times the reference's CPU path of the same linear (its torch restatement in ``oracle/``:
quantize, dequantize, fp32 matmul) on the host cores, on a bounded sample of rows per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent

# Under torchrun (WORLD_SIZE > 1): NCCL's own communicator set-up log (rank count, transports), written per process to
# a file so stdout keeps the one JSON line; rank 0 quotes its "nRanks" lines in the line. Set before torch is imported:
# NCCL reads these variables once, at its first call.
NCCL_LOG = None
if int(os.environ.get("WORLD_SIZE", "1")) > 1 and os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
    NCCL_LOG = f"/tmp/h3b_bench_nccl.{os.getpid()}.log"
    os.environ.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT", NCCL_DEBUG_FILE=NCCL_LOG)
sys.path.insert(0, str(ROOT))

M, N, K = 32768, 13824, 5120
FLOP = 2.0 * M * N * K
WORKLOAD = "BASELINE config 2: NVFP4 linear, X[32768x5120] per-tensor NVFP4 quant + GEMM with W[13824x5120] -> bf16"
METRIC = "NVFP4 DiT-linear TFLOPS (config 2: quant + block-scaled GEMM, 32768x13824x5120)"
# algorithmic bytes of the quantizer (read X, write codes + scales) per step
QUANT_BYTES = M * K * 2 + M * K // 2 + M * K // 16


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": float(d["bf16_tflops"]), "bf16_sustained": float(d.get("bf16_tflops_sustained", 0)),
                "hbm": float(d["hbm_gbs"]), "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def _profile_traffic(name: str) -> float | None:
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt, line 'dram_bytes_per_launch: X')."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every 10 ms while the timed region runs (the
    same fields as nvidia-smi's clocks.sm / clocks_event_reasons.*; reads only, no settings are touched)."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        self._nvml = pynvml
        p = torch.cuda.get_device_properties(self.device_index)
        try:
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.device_index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)

    def _reasons(self) -> int:
        nv = self._nvml
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self._handle))

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append((self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM),
                                     self._reasons()))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        try:
            self._open()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "source": "nvml"}
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml, 10 ms"}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_reference_linear(steps: int, warmup: int, sample_rows: int, threads: int) -> dict:
    """The reference's CPU path of the same linear (oracle restatement): quantize a sample of X rows to NVFP4
    (per-tensor scale of the whole X), dequantize, fp32 matmul against the dequantized weight, round to bf16."""
    import numpy as np
    import torch

    from oracle import quant as oq
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    from cases import outlier_matrix

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    wq, wsf, ws, _, _ = oq.quant_nvfp4_tensor(w.float().numpy())  # offline packing, outside the timing
    w_deq = torch.from_numpy(oq.dequant_nvfp4(wq, wsf, N, K, ws))
    x = outlier_matrix(sample_rows, K, 2, 0.005, 30.0).float().numpy()

    def step():
        q, sf, s, _, _ = oq.quant_nvfp4_tensor(x)
        a = torch.from_numpy(oq.dequant_nvfp4(q, sf, sample_rows, K, s))
        return (a @ w_deq.T).bfloat16()

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    flop = 2.0 * sample_rows * N * K
    return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{sample_rows} of 32768 rows of X per step (quantize + dequantize + fp32 matmul with the "
                      f"dequantized 13824x5120 weight); {steps} steps after {warmup} warm-up",
            "s_per_sample_step": dt}


def run_reference(args) -> None:
    ws, rank, _ = _dist()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    r = cpu_reference_linear(args.steps, args.warmup, sample_rows=256, threads=threads)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["s_per_sample_step"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e2m1", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows_per_step": 256},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def fp8_linear_secondary(ops, dev, stream, args) -> dict:
    """The FP8 linear of BASELINE config 3's QKV projection (32760 x 15360 x 5120): per-token FP8 quantization of a
    bf16 activation + tcgen05 e4m3 GEMM with the row and per-channel scales fused. Reported beside the headline."""
    import torch
    Mf, Nf, Kf = 32760, 15360, 5120
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(Mf, Kf, device=dev, generator=g).bfloat16()
    w = (torch.randn(Nf, Kf, device=dev, generator=g) * 0.02).bfloat16()
    wq, wsc = ops.quantize_fp8_weight(w, "channel")
    del w
    q = torch.empty(Mf, Kf, device=dev, dtype=torch.float8_e4m3fn)
    s = torch.empty(Mf, device=dev)
    y = torch.empty(Mf, Nf, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        ops.quant_fp8_rows(x, q, s)
        ops.gemm_fp8(q, wq, y, scale_a=s, scale_b=wsc)
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 10))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * n)]
    for i in range(n):
        ev[3 * i].record(stream)
        ops.quant_fp8_rows(x, q, s)
        ev[3 * i + 1].record(stream)
        ops.gemm_fp8(q, wq, y, scale_a=s, scale_b=wsc)
        ev[3 * i + 2].record(stream)
    torch.cuda.synchronize()
    qms = sum(ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(n)) / n
    gms = sum(ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(n)) / n
    flop = 2.0 * Mf * Nf * Kf
    del x, q, y, wq
    torch.cuda.empty_cache()
    return {"shape": [Mf, Nf, Kf], "tflops": flop / ((qms + gms) * 1e-3) / 1e12,
            "gemm_tflops": flop / (gms * 1e-3) / 1e12, "gemm_ms": gms, "quant_ms": qms,
            "quant_gbs": (Mf * Kf * 3 + Mf * 4) / (qms * 1e-3) / 1e9}


def vsa_config4_secondary(ops, dev, stream, args) -> dict:
    """Q/K/V bf16 [40, 32768, 128] N(0,1) on an 8x64x64 token grid cut into 4x4x4 tiles (512
    tiles of 64): per-tile E4M3 quantization + tile means (V written as f16 holding its E4M3 values), fp32 tile scores,
    top-32 of 512 per query tile, FP8 VSA fine step on the wide-step kernel (the runner's); the tile kernel's time on
    the same operands beside it. Fine-step algorithmic work 4 * S * (k*64) * D * H = 1.374 TFLOP."""
    import math

    import torch
    H, T, Hh, Ww, D, k = args.vsa_heads, 8, 64, 64, 128, 32
    S = T * Hh * Ww
    n = S // 64
    g = torch.Generator(device=dev).manual_seed(11)
    q, kk, v = (torch.randn(H, S, D, device=dev, generator=g).bfloat16() for _ in range(3))
    grid = torch.arange(S, device=dev).view(T // 4, 4, Hh // 4, 4, Ww // 4, 4)
    perm = grid.permute(0, 2, 4, 1, 3, 5).reshape(-1).to(torch.int32)
    vbs = torch.full((n,), 64, device=dev, dtype=torch.int32)
    tile_row0 = (torch.arange(n, device=dev) * 64).to(torch.int32)
    qb, kb = (torch.empty(H, S, D, device=dev, dtype=torch.uint8) for _ in range(2))
    vb = torch.empty(H, S, D, device=dev, dtype=torch.float16)
    qs, ks, vs = (torch.empty(H, n, device=dev) for _ in range(3))
    vs_head = torch.zeros(H, device=dev)
    qp, kp, vp = (torch.empty(H, n, D, device=dev) for _ in range(3))
    sc = torch.empty(H, n, n, device=dev)
    idx = torch.empty(1, H, n, n, device=dev, dtype=torch.int32)
    num = torch.zeros(1, H, n, device=dev, dtype=torch.int32)
    out = torch.empty(1, H, S, D, device=dev, dtype=torch.bfloat16)
    sm_scale = 1.0 / math.sqrt(D)

    def fine(wide):
        ops.vsa_fp8_ex(qb, kb, vb, out, idx, num, vbs, vbs, vs, vs_head, sm_scale * math.log2(math.e), H, n, n, S, S,
                       qs=qs, ks=ks, idx_ld=n, q_scale_ld=n, kv_scale_ld=n, wide=wide)

    def stages(ev=None):
        marks = [lambda: ops.vsa_tile_quant(q, kk, v, perm, tile_row0, vbs, qb, kb, vb, qs, ks, vs, qp, kp, vp, n,
                                            vs_head=vs_head),
                 lambda: ops.tile_scores(qp, kp, sc, sm_scale),
                 lambda: ops.topk_rows(sc, n, n, 0, [0], [n], [k], idx, num, False),
                 lambda: fine(True)]
        for i, f in enumerate(marks):
            if ev is not None:
                ev[i].record(stream)
            f()
        if ev is not None:
            ev[4].record(stream)

    for _ in range(3):
        stages()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 10))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(reps)]
    for r in range(reps):
        stages(evs[r])
    torch.cuda.synchronize()
    names = ["tile_quant", "tile_scores", "topk", "vsa_fp8"]
    ms = {nm: sum(e[i].elapsed_time(e[i + 1]) for e in evs) / reps for i, nm in enumerate(names)}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fine(False)
    e1.record(stream)
    torch.cuda.synchronize()
    flop = 4.0 * S * (k * 64) * D * H
    total = sum(ms.values())
    res = {"shape": [H, S, D], "k": k, "tiles": n, "ms": ms, "ms_total": total,
           "fine_kernel": "h3b_vsa_fp8_ws (wide step)", "fine_tflops": flop / (ms["vsa_fp8"] * 1e-3) / 1e12,
           "tile_kernel_ms": e0.elapsed_time(e1) / reps,
           "tile_quant_gbs": (3 * H * S * D * 2 + 4 * H * S * D) / (ms["tile_quant"] * 1e-3) / 1e9}
    del q, kk, v, qb, kb, vb, sc, idx, out
    torch.cuda.empty_cache()
    return res


def fp8_chain_secondary(pkg, dev, stream, args) -> dict:
    """the FP8 block chain on 32760 tokens x 5120 (16.145 TFLOP of GEMMs per pass)."""
    import torch
    chain = pkg.runner.Fp8BlockChain.random(dev, seed=13)
    g = torch.Generator(device=dev).manual_seed(17)
    rows = 32760
    x0 = torch.randn(rows, 5120, device=dev, generator=g).bfloat16()
    tabs = (torch.randn(6, 5120, device=dev, generator=g) * 0.1).bfloat16()
    x = x0.clone()
    for _ in range(3):
        x.copy_(x0)
        chain(x, tabs)
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 10))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * n)]
    for i in range(n):
        x.copy_(x0)  # every pass starts from the same stream (the copy is outside the timed interval)
        ev[2 * i].record(stream)
        chain(x, tabs, check=False)
        ev[2 * i + 1].record(stream)
    torch.cuda.synchronize()
    pkg.ops.check_status(dev)  # once after the timed passes
    ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(n)) / n
    flop = chain.flop(rows)
    del chain, x, x0
    torch.cuda.empty_cache()
    return {"rows": rows, "ms": ms, "tflops": flop / (ms * 1e-3) / 1e12, "gemm_tflop": flop / 1e12,
            "launches_per_pass": 8}


def sp_bitexact_check(pkg, dev, ws) -> dict:
    """Two blocks on the (7, 16, 16) latent (32 tiles, 1792 tokens) sequence-parallel over every rank of this job (with
    the runner's default head exchange -- the peer transport where available -- and with NCCL all-to-alls; and with
    the default exchange in the balanced tile order), compared bit for bit with one rank's runner in the same tile order
    on the same input, which every rank also runs on its own GPU. Every step of the sharded block is row-, tile- or
    (head, tile)-local, so the two must agree exactly; the result is the minimum over ranks. Also counts the ranks that
    answer one NCCL all-reduce."""
    import torch
    import torch.distributed as dist
    cfg = pkg.model.DiTConfig(blocks=2, fmt="nvfp4")
    m = pkg.model.DiTModel.random(cfg, device=dev, seed=0)
    grid = (7, 16, 16)
    g = torch.Generator(device=dev).manual_seed(1000)
    x = torch.randn(1, grid[0] * grid[1] * grid[2], cfg.hidden, device=dev, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = pkg.runner.VsaMeta(grid=grid, topk=8)
    refs = {order: pkg.runner.H3FastRunner(m, tile_order=order).forward(x, temb, None, None, meta, context=ctx)
            for order in ("reference", "balanced")}
    flags, transports = [], []
    # the transport the step uses (peer when available), then NCCL, in the reference tile order; then the step's
    # transport in the balanced tile order (the config-5 step's order under sequence parallelism)
    for exchange, order in (("auto", "reference"), ("nccl", "reference"), ("auto", "balanced")):
        if exchange == "nccl" and transports and transports[0] == "nccl":
            continue
        r = pkg.runner.H3FastRunner(m, pkg.sp.SeqParallel(), exchange=exchange, tile_order=order)
        got = r.forward(x, temb, None, None, meta, context=ctx)
        flags.append(1 if torch.equal(got.view(torch.int16), refs[order].view(torch.int16)) else 0)
        transports.append(r.transport if order == "reference" else f"{r.transport}+balanced")
        if ws > 1:
            torch.cuda.synchronize()
            r.close()
    same = torch.tensor(flags, device=dev)
    seen = torch.ones(1, device=dev, dtype=torch.int32)
    if ws > 1:
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        dist.all_reduce(seen)
    del m, x, ctx, refs, got
    torch.cuda.empty_cache()
    return {"sp_bitexact": bool(same.min().item()), "per_transport": dict(zip(transports, map(bool, same.tolist()))),
            "grid": list(grid), "blocks": 2, "ranks_in_nccl_allreduce": int(seen.item()),
            "backend": dist.get_backend() if ws > 1 else None}


def dit_step_secondary(pkg, dev, stream, args, ws) -> dict:
    """one 50-block DiT step on the 31x48x84 latent (124,992 tokens) with cross-attention to 512
    text tokens, NVFP4 linears, FP8 VSA self-attention (top-k of 2016 tiles, --dit-topk: 32 by default), sequence-
    parallel over the ranks of this job (head all-to-all over NCCL). Timed with CUDA events, max over ranks (strong
    scaling: fixed tokens)."""
    import torch
    import torch.distributed as dist
    cfg = pkg.model.DiTConfig(blocks=args.dit_blocks, fmt="nvfp4")
    m = pkg.model.DiTModel.random(cfg, device=dev, seed=0)
    grid = (31, 48, 84)
    S = grid[0] * grid[1] * grid[2]
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(1, S, cfg.hidden, device=dev, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
    temb = m.timestep_embedding(0.5)
    meta = pkg.runner.VsaMeta(grid=grid, topk=args.dit_topk)
    # under sequence parallelism the tiles go in the balanced order (the 3-frame slab's 48-row tiles spread over the
    # ranks instead of filling the last one), the one-GPU denominator in the same order; one GPU alone keeps the
    # reference order (the token-reduction timing pairs tiles in it)
    order = args.dit_tile_order if ws > 1 else "reference"
    reps = max(2, min(args.steps, 3))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    one_gpu = None
    if ws > 1:
        # the denominator of the strong-scaling ratio, in the same job: rank 0 alone runs the step on one GPU (the
        # other ranks wait at the barrier)
        if dist.get_rank() == 0:
            r1 = pkg.runner.H3FastRunner(m, tile_order=order)
            for _ in range(2):
                out = r1.forward(x, temb, None, None, meta, context=ctx)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(reps):
                out = r1.forward(x, temb, None, None, meta, context=ctx)
            e1.record(stream)
            torch.cuda.synchronize()
            one_gpu = e0.elapsed_time(e1) / reps
            del r1, out
            torch.cuda.empty_cache()
        dist.barrier()
    sp = pkg.sp.SeqParallel() if ws > 1 else None
    r = pkg.runner.H3FastRunner(m, sp, exchange=args.dit_exchange, tile_order=order)
    for _ in range(2):
        out = r.forward(x, temb, None, None, meta, context=ctx)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        out = r.forward(x, temb, None, None, meta, context=ctx)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    exchange = None
    if ws > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
        # one more step with device events around every exchange on the compute stream: per-kind time per step (max
        # over ranks). NCCL: each all-to-all, waiting for the slowest rank included. Peer transport: the bounded waits
        # for the peers' flags, i.e. the exchange time left exposed after the copies overlapped the attention
        r.ex.timing = []
        out = r.forward(x, temb, None, None, meta, context=ctx)
        torch.cuda.synchronize()
        names = (["wait_tile_stats", "wait_qkv", "wait_attn_out"] if r.transport == "peer" else
                 ["qkv_e4m3", "tile_stats", "attn_out_bf16"])
        per = {nm: 0.0 for nm in names}
        for nm, a, b in r.ex.timing:
            per[nm] += a.elapsed_time(b)
        r.ex.timing = None
        t = torch.tensor([per[nm] for nm in names], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        exchange = {"transport": r.transport, "head_groups": r.head_groups, "ms_per_step": dict(zip(names, t.tolist())),
                    "note": ("time the compute stream waited for the peers' flags (Q/K/V and outputs copied by the "
                             "copy engines into peer-mapped buffers while attention ran), summed over the blocks of "
                             "one step, max over ranks" if r.transport == "peer" else
                             "device time of each kind of all-to-all summed over the blocks of one step (max over "
                             "ranks); each exchange includes waiting for the slowest rank to reach it")}
        if r.transport_note:
            exchange["peer_unavailable"] = r.transport_note[:300]
        dist.barrier()
        if r.transport == "peer" and not args.no_nccl_compare:
            # the same step with the NCCL all-to-all transport (all heads at once, no overlap), same job
            try:
                rn = pkg.runner.H3FastRunner(m, sp, exchange="nccl", tile_order=order)
                for _ in range(2):
                    out = rn.forward(x, temb, None, None, meta, context=ctx)
                torch.cuda.synchronize()
                dist.barrier()
                e0.record(stream)
                for _ in range(reps):
                    out = rn.forward(x, temb, None, None, meta, context=ctx)
                e1.record(stream)
                torch.cuda.synchronize()
                t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                exchange["nccl_transport_ms_per_step"] = float(t.item())
            except Exception as exc:  # an extra timing must not cost the line; its error is reported
                exchange["nccl_transport_error"] = repr(exc)[:300]
            finally:
                rn = None
                torch.cuda.empty_cache()
            dist.barrier()
    finite = bool(torch.isfinite(out.float()).all())
    reduced = None
    if args.dit_extras and ws == 1 and not args.dit_reduction:
        args.dit_reduction = "4:30"  # the reference schedule's default interval (blocks 4..29)
    if args.dit_reduction and ws == 1:
        try:
            # token reduction (one rank, like the reference runner): blocks [begin, end) on horizontally paired tokens
            parts = args.dit_reduction.split(":")
            b, e = int(parts[0]), int(parts[1])
            scale = float(parts[2]) if len(parts) > 2 else 1.0
            plan = pkg.reduction.build_token_reduction(grid, b, min(e, cfg.blocks), scale)
            for _ in range(2):
                out = r.forward(x, temb, None, None, meta, context=ctx, reduction=plan)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(reps):
                out = r.forward(x, temb, None, None, meta, context=ctx, reduction=plan)
            e1.record(stream)
            torch.cuda.synchronize()
            reduced = {"blocks": [b, min(e, cfg.blocks)], "update_scale": scale,
                       "reduced_grid": list(plan.reduced_grid), "ms_per_step": e0.elapsed_time(e1) / reps,
                       "output_finite": bool(torch.isfinite(out.float()).all())}
        except Exception as exc:  # an extra timing must not cost the line; its error is reported
            reduced = {"error": repr(exc)[:300]}
            torch.cuda.empty_cache()
    graphed = None
    if args.dit_graph and ws == 1:
        # the same step replayed from one CUDA graph (every launch of the 50 blocks captured once)
        gf = pkg.runner.GraphedForward(r, x, temb, meta, ctx)
        for _ in range(2):
            out = gf(x, temb)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            out = gf(x, temb)
        e1.record(stream)
        torch.cuda.synchronize()
        graphed = {"ms_per_step": e0.elapsed_time(e1) / reps, "output_finite": bool(torch.isfinite(out.float()).all())}
        del gf
    qk8 = None
    r8 = None
    if args.dit_qk_int8 or (args.dit_extras and ws == 1):
        try:
            # the same step with INT8 QK^T in the self-attention (tcgen05 kind::i8 scores)
            r8 = pkg.runner.H3FastRunner(m, sp, qk_int8=True, tile_order=order)
            for _ in range(2):
                out = r8.forward(x, temb, None, None, meta, context=ctx)
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            e0.record(stream)
            for _ in range(reps):
                out = r8.forward(x, temb, None, None, meta, context=ctx)
            e1.record(stream)
            torch.cuda.synchronize()
            t8 = e0.elapsed_time(e1) / reps
            if ws > 1:
                t = torch.tensor([t8], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                t8 = float(t.item())
            qk8 = {"ms_per_step": t8, "output_finite": bool(torch.isfinite(out.float()).all())}
        except Exception as exc:  # an extra timing must not cost the line; its error is reported
            qk8 = {"error": repr(exc)[:300]}
            try:
                torch.cuda.synchronize()
            except Exception:  # noqa: BLE001  a sticky CUDA error: every later GPU line would fail for this reason
                qk8["context_lost"] = True
        finally:
            r8 = None
            torch.cuda.empty_cache()
    ffn_static = None
    if args.dit_ffn_static or (args.dit_extras and ws == 1):
        try:
            # the same step with the FFN intermediate re-quantized in fc_in's epilogue under fixed per-block global
            # scales (recorded by the first forward) instead of the bf16 store + per-row quantization pass
            rs = pkg.runner.H3FastRunner(m, sp, ffn_requant="static", tile_order=order)
            for _ in range(2):
                out = rs.forward(x, temb, None, None, meta, context=ctx)
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            e0.record(stream)
            for _ in range(reps):
                out = rs.forward(x, temb, None, None, meta, context=ctx)
            e1.record(stream)
            torch.cuda.synchronize()
            tf = e0.elapsed_time(e1) / reps
            if ws > 1:
                t = torch.tensor([tf], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                tf = float(t.item())
            ffn_static = {"ms_per_step": tf, "output_finite": bool(torch.isfinite(out.float()).all()),
                          "headroom": rs.ffn_headroom}
        except Exception as exc:  # an extra timing must not cost the line; its error is reported
            ffn_static = {"error": repr(exc)[:300]}
            try:
                torch.cuda.synchronize()
            except Exception:  # noqa: BLE001  a sticky CUDA error: every later GPU line would fail for this reason
                ffn_static["context_lost"] = True
        finally:
            rs = None
            torch.cuda.empty_cache()
    lin = 2.0 * S * (6 * cfg.hidden ** 2 + 2 * cfg.hidden * cfg.ffn) * cfg.blocks
    if ws > 1:
        r.close()
    del r, m, x, out
    torch.cuda.empty_cache()
    res = {"grid": list(grid), "tokens": S, "blocks": cfg.blocks, "topk": args.dit_topk, "n_gpus": ws,
           "ms_per_step": ms, "steps": reps, "linear_tflop_per_step": lin / 1e12,
           "linear_share_tflops": lin / (ms * 1e-3) / 1e12, "output_finite": finite, "scaling": "strong",
           "parallelism": f"sp{ws}", "tile_order": order}
    if one_gpu is not None:
        res["one_gpu_ms_per_step_same_job"] = one_gpu
    if exchange is not None:
        res["exchanges"] = exchange
    if reduced is not None:
        res["token_reduction"] = reduced
    if qk8 is not None:
        res["qk_int8"] = qk8
    if ffn_static is not None:
        res["ffn_static_requant"] = ffn_static
    if graphed is not None:
        res["cuda_graph"] = graphed
    return res


def memory_kernels_secondary(pkg, dev, args) -> dict:
    """The memory-bound kernels of the path, each at its BASELINE size (``--mem-rows`` overrides the row counts): the
    per-tensor NVFP4 quantizer of config 2 (amax pass and quantize pass), the LayerNorm + modulate + NVFP4 quantizer and
    the q/k/v prologue of the config-5 block (124,992 rows), the per-row NVFP4 quantizer of the FFN intermediate
    (13824 wide), the attention-output gate quantizer and the tile selection (top-32 of 2016). Median of ``reps``
    launches (CUDA events) after warm-ups; GB/s are algorithmic bytes (inputs read once, outputs written once) over
    the launch time, and ``frac`` divides them by the measured HBM copy bandwidth."""
    import torch
    ops = pkg.ops
    reps, warm = (1, 0) if args.mem_once else (10, 3)
    hbm = _peaks()["hbm"]
    g = torch.Generator(device=dev).manual_seed(31)

    def tm(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    out = {}

    def rec(name, ms, nbytes, note):
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "alg_bytes": nbytes, "gbs": gbs, "frac": gbs / hbm, "what": note}

    M2, K = (args.mem_rows or 32768), 5120
    x = torch.randn(M2, K, device=dev, generator=g).bfloat16()
    q = torch.empty(M2, K // 2, device=dev, dtype=torch.uint8)
    sf = torch.empty(ops.sf_rows(M2), K // 16, device=dev, dtype=torch.uint8)
    s, am = torch.empty(1, device=dev), torch.zeros(1, device=dev)
    rec("amax_c2", tm(lambda: ops.amax(x, am)), M2 * K * 2, f"amax pass over X [{M2} x {K}] bf16")
    rec("quant_nvfp4_tensor_c2", tm(lambda: ops.quant_nvfp4_tensor(x, am, q, sf, s)),
        M2 * K * 2 + M2 * (K // 2 + K // 16), "quantize pass: read X, write codes + block scales")
    del x, q, sf
    R = args.mem_rows or 124992
    xl = torch.randn(R, K, device=dev, generator=g).bfloat16()
    tabs = (torch.randn(2, K, device=dev, generator=g) * 0.1).bfloat16()
    h = torch.empty(R, K // 2, device=dev, dtype=torch.uint8)
    hsf = torch.zeros(ops.sf_rows(R), K // 16, device=dev, dtype=torch.uint8)
    hs = torch.empty(R, device=dev)
    rec("layer_norm_quant_c5", tm(lambda: ops.resid_norm_quant(xl, None, None, None, None, None, tabs[0:1], tabs[1:2],
                                                                 xl, h, hsf, hs, 1e-6, norm="layer")),
        R * K * 2 + R * (K // 2 + K // 16 + 4), f"LayerNorm + modulate + NVFP4, {R} x {K}")
    del xl, h, hsf, hs
    F = 13824
    Rf = min(R, 32768)
    u = torch.randn(Rf, F, device=dev, generator=g).bfloat16()
    f = torch.empty(Rf, F // 2, device=dev, dtype=torch.uint8)
    fsf = torch.zeros(ops.sf_rows(Rf), F // 16, device=dev, dtype=torch.uint8)
    fs = torch.empty(Rf, device=dev)
    rec("quant_nvfp4_rows_ffn", tm(lambda: ops.quant_nvfp4_rows(u, f, fsf, fs)), Rf * F * 2 + Rf * (F // 2 + F // 16 + 4),
        f"per-row NVFP4 of the FFN intermediate, {Rf} x {F}")
    del u, f, fsf
    H, n = 40, (R // 64) - (R // 64) % 2
    rows = n * 64
    qkv = torch.randn(rows, 3 * K, device=dev, generator=g).bfloat16()
    s1 = torch.rand(rows, device=dev, generator=g) + 0.5
    wq, wk = (torch.randn(128, device=dev, generator=g).bfloat16() for _ in range(2))
    ang = torch.rand(rows, 48, device=dev, generator=g) * 6.28
    cos, sin = torch.cat([ang.cos()] * 2, -1).bfloat16(), torch.cat([ang.sin()] * 2, -1).bfloat16()
    vbs = torch.full((n,), 64, device=dev, dtype=torch.int32)
    row0 = torch.arange(n, device=dev, dtype=torch.int32) * 64
    qb, kb, vb = (torch.zeros(H, rows, 128, device=dev, dtype=torch.uint8) for _ in range(3))
    qs, ks, vs = (torch.ones(H, n, device=dev) for _ in range(3))
    qp, kp, vp = (torch.zeros(H, n, 128, device=dev) for _ in range(3))
    rec("qkv_prologue_c5", tm(lambda: ops.qkv_prologue8(qkv[:, :K], qkv[:, K:2 * K], qkv[:, 2 * K:], s1, row0, vbs, wq, wk,
                                                        cos, sin, 1.0, 1.0, qb, kb, vb, vs, None, qp, kp, vp, H, n, 64,
                                                        1e-6, qs_blk=qs, ks_blk=ks)),
        3 * rows * K * 2 + 3 * rows * K + 3 * H * n * 128 * 4, f"q/k/v prologue, {H} heads x {rows} rows")
    ob = torch.randn(H, rows, 128, device=dev, generator=g).bfloat16()
    slot = torch.arange(rows, device=dev, dtype=torch.int32)
    a = torch.empty(rows, K // 2, device=dev, dtype=torch.uint8)
    asf = torch.zeros(ops.sf_rows(rows), K // 16, device=dev, dtype=torch.uint8)
    sa = torch.empty(rows, device=dev)
    rec("attn_gate_quant_c5", tm(lambda: ops.attn_gate_quant(ob, None, None, None, slot, n, 64, a, asf, sa, rows)),
        rows * K * 2 + rows * (K // 2 + K // 16 + 4), f"attention output gather + NVFP4, {rows} rows")
    del qkv, qb, kb, vb, ob, a, asf
    nt = 2016 if not args.mem_rows else max(64, min(2016, (args.mem_rows // 64) // 2 * 2))
    sc = torch.randn(H, nt, nt, device=dev, generator=g)
    idx = torch.empty(1, H, nt, nt, device=dev, dtype=torch.int32)
    num = torch.zeros(1, H, nt, device=dev, dtype=torch.int32)
    rec("topk_select_c5", tm(lambda: ops.topk_rows(sc, nt, nt, 0, [0], [nt], [32], idx, num, False)),
        H * nt * nt * 4 + H * nt * 32 * 4, f"top-32 of {nt} tiles, {H} heads")
    del sc, idx
    torch.cuda.empty_cache()
    out["hbm_peak_gbs"] = hbm
    return out


def run_only(args) -> None:
    """One secondary measurement alone (for profiling captures): prints its JSON object."""
    import torch
    import torch.distributed as dist

    import __graft_entry__
    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    pkg = __graft_entry__.load_package()
    stream = torch.cuda.current_stream(dev)
    fn = {"fp8": lambda: fp8_linear_secondary(pkg.ops, dev, stream, args),
          "chain": lambda: fp8_chain_secondary(pkg, dev, stream, args),
          "vsa": lambda: vsa_config4_secondary(pkg.ops, dev, stream, args),
          "dit": lambda: dit_step_secondary(pkg, dev, stream, args, ws),
          "mem": lambda: memory_kernels_secondary(pkg, dev, args)}[args.only]
    res = fn()
    if rank == 0:
        print(json.dumps({"only": args.only, "n_gpus": ws, "result": res}), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def weight_pack_secondary(ops, w, dev) -> dict:
    """Offline NVFP4 packing of the config-2 weight W [13824 x 5120] (amax pass + e2m1/ue4m3 pack), CUDA events over
    5 launches after 2 warm-ups; algorithmic bytes: read W once (bf16), write codes + block scales."""
    import torch
    wsp = torch.empty(256, device=dev, dtype=torch.uint8)
    outs = [torch.empty(N, K // 2, device=dev, dtype=torch.uint8),
            torch.empty(N, K // 16, device=dev, dtype=torch.uint8), torch.empty(1, device=dev)]
    lib_call = ops.call
    stream = torch.cuda.current_stream(dev)

    def once():
        lib_call("h3b_pack_weight_nvfp4", w.data_ptr(), N, K, outs[0].data_ptr(), outs[1].data_ptr(),
                 outs[2].data_ptr(), wsp.data_ptr(), stream.cuda_stream)

    for _ in range(2):
        once()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        once()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 5
    alg = N * K * 2 + N * K // 2 + N * K // 16
    return {"shape": [N, K], "ms": ms, "alg_bytes": alg, "gbs": alg / (ms * 1e-3) / 1e9,
            "note": "amax pass + pack; the amax pass reads W a second time (not counted)"}


def e2e_pipelined(ops, x_host, qw, sfw, sw, dev, args, barrier) -> tuple[float, int]:
    """End to end through the public ops with the host copies overlapped: step i's input copy (host -> device, its own
    stream), step i-1's quantize + GEMM and step i-2's result copy (device -> host, its own stream) run at once on
    double-buffered device and pinned host buffers; PCIe carries both directions at the same time. Every step still
    moves its own 335 MB in and 906 MB out. Device-timed from the first input copy to the last result copy."""
    import torch
    bf = torch.bfloat16
    xs = [torch.empty(M, K, device=dev, dtype=bf) for _ in range(2)]
    ys = [torch.empty(M, N, device=dev, dtype=bf) for _ in range(2)]
    y_hosts = [torch.empty(M, N, dtype=bf).pin_memory() for _ in range(2)]
    qa = torch.empty(M, K // 2, device=dev, dtype=torch.uint8)
    sfa = torch.empty(ops.sf_rows(M), K // 16, device=dev, dtype=torch.uint8)
    sa = torch.empty(1, device=dev)
    wsp = torch.empty(ops.workspace_bytes(), device=dev, dtype=torch.uint8)
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def one(i: int) -> None:
        b = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[b])  # step i-2 has read xs[b]
            xs[b].copy_(x_host, non_blocking=True)
            ev_in[b].record(s_in)
        comp.wait_event(ev_in[b])
        if i >= 2:
            comp.wait_event(ev_out[b])  # step i-2's result has left ys[b]
        ops.quant_nvfp4(xs[b], qa, sfa, sa, wsp)
        ops.gemm_nvfp4(qa, sfa, qw, sfw, ys[b], alpha_dev=sa, scale_b=sw)
        ev_comp[b].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            y_hosts[b].copy_(ys[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(2):
        one(i)
    torch.cuda.synchronize()
    barrier()
    steps = max(4, min(args.steps, 8))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(steps):
        one(2 + i)
    t1.record(s_out)
    torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1) / steps
    del xs, ys, y_hosts
    torch.cuda.empty_cache()
    return ms, steps


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import __graft_entry__
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    from cases import outlier_matrix

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    ops = __graft_entry__.load_package().ops

    # inputs: X on the host (pinned, for the end-to-end leg) and resident in HBM; the packed weight
    x_host = outlier_matrix(M, K, 2 + rank, 0.005, 30.0).pin_memory()
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(3)) * 0.02).bfloat16().to(dev)
    qw, sfw, sw = ops.pack_nvfp4_weight(w)
    pack = weight_pack_secondary(ops, w, dev)
    del w
    x = x_host.to(dev)
    qa = torch.empty(M, K // 2, device=dev, dtype=torch.uint8)
    sfa = torch.empty(ops.sf_rows(M), K // 16, device=dev, dtype=torch.uint8)
    sa = torch.empty(1, device=dev)
    wsp = torch.empty(ops.workspace_bytes(), device=dev, dtype=torch.uint8)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    y_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream(dev)
    launches_per_step = 3  # amax, NVFP4 quantizer, GEMM

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        ops.quant_nvfp4(x, qa, sfa, sa, wsp)
        if ev is not None:
            ev[1].record(stream)
        ops.gemm_nvfp4(qa, sfa, qw, sfw, y, alpha_dev=sa, scale_b=sw)
        if ev is not None:
            ev[2].record(stream)

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t_start.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ops.check_status(dev)  # a GEMM whose bounded wait expired during the timed steps fails the run
    total_ms = t_start.elapsed_time(t_end)
    quant_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    gemm_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps

    # end to end through the public ops: pinned host X -> device, quantize + GEMM, Y -> pinned host, every step
    for _ in range(max(1, args.warmup // 2)):
        x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 5))
    e0.record(stream)
    for _ in range(e2e_steps):
        x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_serial_ms = e0.elapsed_time(e1) / e2e_steps
    e2e_ms, e2e_steps_p = e2e_pipelined(ops, x_host, qw, sfw, sw, dev, args, barrier)

    pkg = __graft_entry__.load_package()
    fp8 = fp8_linear_secondary(ops, dev, stream, args) if not args.no_fp8 else None
    chain = fp8_chain_secondary(pkg, dev, stream, args) if not args.no_fp8 else None
    vsa = vsa_config4_secondary(ops, dev, stream, args) if not args.no_vsa else None
    del x, y, qa, sfa
    torch.cuda.empty_cache()
    sp_check = sp_bitexact_check(pkg, dev, ws) if ws > 1 else None
    mem = memory_kernels_secondary(pkg, dev, args) if ws == 1 and not args.no_mem else None
    dit = dit_step_secondary(pkg, dev, stream, args, ws) if not args.no_dit else None

    if ws > 1:
        t = torch.tensor([total_ms, e2e_ms, gemm_ms, quant_ms, e2e_serial_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms, gemm_ms, quant_ms, e2e_serial_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    value = ws * FLOP / (ms_per_step * 1e-3) / 1e12

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_reference_linear(steps=3, warmup=1, sample_rows=256, threads=os.cpu_count() or 1)
        cpu.pop("s_per_sample_step", None)

    if rank == 0:
        peaks = _peaks()
        fp4_peak = 4.0 * peaks["bf16"]  # dense FP4 runs at 4x dense bf16 on B200; 4 x the measured bf16 figure
        gemm_tflops = FLOP / (gemm_ms * 1e-3) / 1e12
        traffic = _profile_traffic("gemm_nvfp4_config2")
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": M, "N": N, "K": K, "parallelism": f"dp{ws}",
                       "l2": "inputs larger than L2 (X 335 MB read, Y 906 MB written per step); no flush"},
            "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": fp4_peak, "unit": "TFLOP/s",
                         "frac": gemm_tflops / fp4_peak, "traffic": traffic,
                         "kernel": "gemm_nvfp4_pair_kernel (CTA pair, 256x192 tiles, tcgen05 mxf4nvf4 block16)",
                         "peak_source": f"4 x {peaks['source']} dense bf16 ({peaks['bf16']} TFLOP/s)",
                         "nominal_peak": 9000.0},
            "kernels_ms": {"nvfp4_quant_incl_amax": quant_ms, "gemm": gemm_ms,
                           "quant_gbs": QUANT_BYTES / (quant_ms * 1e-3) / 1e9, "hbm_peak_gbs": peaks["hbm"]},
            "e2e": {"value": ws * FLOP / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2, "ms_per_step": e2e_ms,
                    "steps": e2e_steps_p, "copies": "overlapped: input copy, compute and result copy of consecutive "
                    "steps on three streams, double-buffered",
                    "serial_ms_per_step": e2e_serial_ms},
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
        }
        pack["frac_of_hbm"] = pack["gbs"] / peaks["hbm"]
        line["weight_pack_nvfp4"] = pack
        if fp8 is not None:
            fp8["gemm_frac_of_2x_bf16"] = fp8["gemm_tflops"] / (2.0 * peaks["bf16"])
            line["fp8_linear"] = fp8
        if vsa is not None:
            vsa["fine_frac_of_2x_bf16"] = vsa["fine_tflops"] / (2.0 * peaks["bf16"])
            line["vsa_config4"] = vsa
        if chain is not None:
            chain["frac_of_2x_bf16"] = chain["tflops"] / (2.0 * peaks["bf16"])
            line["fp8_block_chain_config3"] = chain
        if sp_check is not None:
            line["sp_check"] = sp_check
        if NCCL_LOG is not None:
            try:
                with open(NCCL_LOG) as fh:
                    init = [ln.strip() for ln in fh if "nRanks" in ln or "NCCL version" in ln]
                line["nccl_init_log"] = {"file": NCCL_LOG, "lines": init[:4]}
            except OSError as exc:
                line["nccl_init_log"] = {"file": NCCL_LOG, "error": repr(exc)[:200]}
        if mem is not None:
            line["memory_kernels"] = mem
        if dit is not None:
            line["dit_step_config5"] = dit
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--dit-graph", action="store_true",
                    help="also time the config-5 step replayed from one CUDA graph (one GPU)")
    ap.add_argument("--no-dit-extras", dest="dit_extras", action="store_false",
                    help="skip the one-GPU extra config-5 timings run by default: token reduction over blocks 4..29, "
                         "INT8 QK^T and the static FFN re-quantization")
    ap.add_argument("--dit-qk-int8", action="store_true",
                    help="also time the config-5 step with INT8 QK^T in the self-attention")
    ap.add_argument("--dit-ffn-static", action="store_true",
                    help="also time the config-5 step with the FFN re-quantized in fc_in's epilogue (static scales)")
    ap.add_argument("--dit-exchange", choices=["auto", "peer", "nccl"], default="auto",
                    help="head exchange of the sequence-parallel config-5 step: peer-mapped buffers written by the "
                         "copy engines with head groups pipelined behind the attention (auto: when every rank maps "
                         "every other's memory), or NCCL all-to-alls")
    ap.add_argument("--dit-tile-order", choices=["balanced", "reference"], default="balanced",
                    help="tile order of the sequence-parallel config-5 step (N > 1): balanced (the edge tiles spread "
                         "evenly over the ranks' shards) or the reference's (t, h, w) order")
    ap.add_argument("--no-nccl-compare", action="store_true",
                    help="with the peer transport, skip timing the same config-5 step over NCCL in the same job")
    ap.add_argument("--dit-reduction", default="", metavar="BEGIN:END[:SCALE]",
                    help="also time the config-5 step with token reduction over blocks [BEGIN, END) (one GPU)")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-fp8", action="store_true", help="skip the secondary FP8 linear measurement")
    ap.add_argument("--no-vsa", action="store_true", help="skip the secondary VSA (config 4) measurement")
    ap.add_argument("--no-dit", action="store_true", help="skip the secondary 50-block DiT step (config 5)")
    ap.add_argument("--no-mem", action="store_true", help="skip the memory-bound kernel measurements")
    ap.add_argument("--mem-rows", type=int, default=0,
                    help="row count of the memory-kernel measurements (0: BASELINE sizes; smaller for ncu captures)")
    ap.add_argument("--mem-once", action="store_true",
                    help="memory kernels: one launch each, no warm-up (so an ncu capture sees each kernel once)")
    ap.add_argument("--only", choices=["fp8", "chain", "vsa", "dit", "mem"], default=None,
                    help="run one secondary measurement alone (profiling captures); no headline line")
    ap.add_argument("--vsa-heads", type=int, default=40, help="heads of the config-4 VSA measurement (40)")
    ap.add_argument("--dit-blocks", type=int, default=50, help="blocks of the config-5 step (50)")
    ap.add_argument("--dit-topk", type=int, default=32,
                    help="key tiles per query tile in the config-5 step (32, C4's density; 404 = the reference's 0.8 "
                         "sparsity over 2016 tiles)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
