"""The bench's output contract on the CPU: ``bench.py --impl reference`` (the reference arm: the CPU restatement timed
on the host cores) prints one JSON line with the keys the benchmark driver reads, and the same metric/unit as the
GPU arm; argument parsing accepts the GPU arm's options."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup",
                        "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("BASELINE config 2")
    import bench
    assert d["metric"] == bench.METRIC


def test_arguments_of_both_arms_parse():
    import bench
    ap_help = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                             timeout=120, cwd=ROOT)
    assert ap_help.returncode == 0
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--dit-reduction", "--dit-qk-int8", "--dit-graph",
                "--dit-topk"):
        assert opt in ap_help.stdout, opt
    assert bench.FLOP == 2.0 * 32768 * 13824 * 5120
