"""Vocabulary sharding over NCCL on real GPUs: the sharded tokens equal the single-GPU
tokens bit for bit (needs at least 2 GPUs; skipped on a 1-GPU box).

The check runs as 2 (or, with DELS_NCCL_TEST_RANKS, more) torch.distributed.run ranks
of tests/sharded_nccl_worker.py, one per GPU, at the full vocabulary-sharded size."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_nccl_vocab_shards_match_single_gpu(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    n = min(int(os.environ.get("DELS_NCCL_TEST_RANKS", "2")), torch.cuda.device_count())
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out = tmp_path / "verdict.json"
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(n), "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(ROOT / "tests" / "sharded_nccl_worker.py"), "--out", str(out)]
    proc = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-3000:]
    v = json.loads(out.read_text())
    assert v["world"] == n and v["rows"] == 16384
    assert v["tokens_equal"] and v["scores_equal"] and v["gathered_tokens_equal"], v
