"""bench.py's one-line JSON contract, checked on the host: the reference arm (the
reference formula in torch on the CPU) runs without a GPU and prints every key the
driver reads, with our arm's metric, unit and workload config.  CPU only."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
BASELINE = json.loads((ROOT / "BASELINE.json").read_text()) if (ROOT / "BASELINE.json").exists() else {}


def test_reference_arm_line_on_the_host():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=900, check=True, cwd=ROOT).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1, out
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["unit"] == "rows/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "cfg2_qwen3_8b_bf16_b32x16" and d["config"]["rows"] == 512
    assert d["dtype"] == "bf16"
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    if "metric" in BASELINE:
        assert d["metric"] == BASELINE["metric"]


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the driver's N > 1 runs: rank 0 alone times the reference formula on
    the sharded workload's config and prints one line; every rank exits 0."""
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    proc = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                           "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
                           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"],
                          capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1, proc.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["scaling"] == "strong"
    assert d["config"]["workload"] == "cfg5_vocab_sharded_16384" and d["value"] > 0
