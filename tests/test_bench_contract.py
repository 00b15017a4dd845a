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


def _bench():
    import importlib.util

    spec = importlib.util.spec_from_file_location("dels_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_default_workload_follows_the_launcher(monkeypatch):
    """A plain run times the 512-row headline; under torch.distributed.run every N, N = 1
    included, times the vocabulary-sharded 16384-row workload, so a 1/2/4/8 scaling
    series compares one workload."""
    b = _bench()
    for var in ("TORCHELASTIC_RUN_ID", "LOCAL_WORLD_SIZE"):
        monkeypatch.delenv(var, raising=False)
    assert b.default_workload(1) == "cfg2"
    assert b.default_workload(2) == "cfg5"
    monkeypatch.setenv("TORCHELASTIC_RUN_ID", "none")
    assert b.default_workload(1) == "cfg5"
    cfg1 = b.dense_config("cfg5_vocab_sharded_16384", 16384, 4096, 256, 151936, 1, True)
    cfg8 = b.dense_config("cfg5_vocab_sharded_16384", 16384, 4096, 256, 151936, 8, True)
    assert cfg1["parallelism"] == "vocab-shard x1" and cfg1["vocab_per_rank"] == 151936
    assert cfg8["parallelism"] == "vocab-shard x8" and cfg8["vocab_per_rank"] == 19200
    assert {k: v for k, v in cfg1.items() if k not in ("parallelism", "vocab_per_rank")} == \
        {k: v for k, v in cfg8.items() if k not in ("parallelism", "vocab_per_rank")}


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
    # exactly the dict our arm prints for the same workload (the driver compares them)
    assert d["config"] == _bench().dense_config("cfg2_qwen3_8b_bf16_b32x16", 512, 4096, 256, 151936, 1, False)
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
    assert d["config"] == _bench().dense_config("cfg5_vocab_sharded_16384", 16384, 4096, 256, 151936, 2, True)


def test_reference_arm_markov_on_the_host():
    """The Markov runner workload's reference arm: the reference runner's torch rollout on the
    host, with the config dict our arm prints."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "markov",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=900, check=True,
                         cwd=ROOT).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1, out
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "rows/s" and d["value"] > 0
    assert d["config"] == {"workload": "markov_b1_steps14", "V": 151936, "r": 256,
                           "note": "one step = one MarkovDeLSGraphRunner call (14 scored positions per sequence)"}
    assert d["cpu_baseline"]["value"] == d["value"] and "rollout" in d["cpu_baseline"]["sample"]
