"""Benchmark of the B200 quantized DiT-linear hot path (BASELINE.json metric "NVFP4/FP8 DiT-linear TFLOPS").

Workload (the configuration the metric is quoted on): one NVFP4 DiT linear per step --
X bf16 [32768 x 5120] (N(0,1), 0.5% of columns x30) -> per-tensor NVFP4 quantization (amax pass + e2m1/ue4m3 pack)
-> block-scaled tcgen05 GEMM with the pre-packed weight W [13824 x 5120] -> Y bf16 [32768 x 13824].
2*M*N*K = 4.638 TFLOP per step. Inputs (X 335 MB) and outputs (Y 906 MB) are larger than the 126 MB L2, so no flush.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; each rank processes its own 32768-token shard (weak scaling, no data
collective: the linear is row-independent). Rank 0 prints one JSON line.
``--impl reference`` times the reference's CPU path of the same linear (its torch restatement in ``oracle/``:
quantize, dequantize, fp32 matmul) on the host cores, on a bounded sample of rows per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
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
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


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
    e2e_ms = e0.elapsed_time(e1) / e2e_steps

    if ws > 1:
        t = torch.tensor([total_ms, e2e_ms, gemm_ms, quant_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms, gemm_ms, quant_ms = t.tolist()
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
                         "kernel": "gemm_kernel<FP4=true,BN=192> (tcgen05 mxf4nvf4 block16)",
                         "peak_source": f"4 x {peaks['source']} dense bf16 ({peaks['bf16']} TFLOP/s)",
                         "nominal_peak": 9000.0},
            "kernels_ms": {"nvfp4_quant_incl_amax": quant_ms, "gemm": gemm_ms,
                           "quant_gbs": QUANT_BYTES / (quant_ms * 1e-3) / 1e9, "hbm_peak_gbs": peaks["hbm"]},
            "e2e": {"value": ws * FLOP / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2, "ms_per_step": e2e_ms},
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
