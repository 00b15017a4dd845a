"""Vocab-sharded (max, index) combine on CPU ranks (gloo): per-rank oracle keys over a
vocabulary slice, all-reduce(MAX), decode == the unsharded argmax, including ties that
straddle shard boundaries; and a rank that fails before the combine makes the others'
collective fail instead of hang.  No GPU."""

from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(V: int):
    from oracle import dels_oracle as O

    rng = np.random.default_rng(123)
    rows, H, r = 12, 32, 8
    h = O.bf16_round(rng.standard_normal((rows, H)).astype(np.float32))
    W = O.bf16_round((rng.standard_normal((V, H)) * 0.1).astype(np.float32))
    Ut = O.bf16_round((rng.standard_normal((r, H)) * 0.1).astype(np.float32))
    Vr = O.bf16_round((rng.standard_normal((V, r)) * 0.1).astype(np.float32))
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    # Planted exact ties across shards: rows 0-2 see the same huge score at tokens
    # 1 and V-2 (first and last shard); row 3 sees all-zero logits and no prior.
    W[1] = 0
    W[V - 2] = 0
    W[1, 0] = W[V - 2, 0] = 8.0
    Vr[1] = Vr[V - 2] = 0
    prior[1] = prior[V - 2] = 0.0
    h[0:3, 0] = 4.0
    return h, W, Ut, Vr, prior


def _worker(rank, world, port, V, q, fail_rank):
    try:
        sys.path[:0] = [str(ROOT), str(ROOT / "dels-spec_b200")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        from dels_b200 import sharded, workloads
        from oracle import dels_oracle as O

        h, W, Ut, Vr, prior = _case(V)
        alpha, beta = np.linspace(0.5, 0.1, 4), np.linspace(0.3, 0.0, 4)
        v0, v1 = workloads.shard_range(V, world, rank, align=64)
        _, sc, _ = O.draft_score_bf16(h, W[v0:v1], Ut, Vr[v0:v1], prior[v0:v1], alpha, beta, n_pos=4)
        local = np.argmax(sc, axis=1)
        keys = torch.from_numpy(O.pack_keys(sc[np.arange(len(local)), local].astype(np.float32), local + v0))
        if rank == fail_rank:
            raise RuntimeError("planted failure before the combine")
        sharded.combine_keys(keys)
        tok, score = sharded.decode_keys_host(keys)
        q.put((rank, "ok", tok.numpy(), score.numpy()))
    except Exception as exc:  # reported to the parent
        q.put((rank, "error", repr(exc), traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, V, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, V, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, a, b = q.get(timeout=120)
        results[rank] = (status, a, b)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_combine_equals_unsharded(world):
    from oracle import dels_oracle as O

    V = 997
    res = _run(world, V)
    h, W, Ut, Vr, prior = _case(V)
    tok, sc, gap = O.draft_score_bf16(h, W, Ut, Vr, prior, np.linspace(0.5, 0.1, 4), np.linspace(0.3, 0.0, 4),
                                      n_pos=4)
    for rank in range(world):
        status, got, score = res[rank]
        assert status == "ok", got
        np.testing.assert_array_equal(got, tok)  # identical on every rank, ties -> lowest index
        np.testing.assert_allclose(score, sc[np.arange(len(tok)), tok], rtol=0, atol=1e-5)
    assert list(tok[:3]) == [1, 1, 1]  # the planted cross-shard tie went to the lower token


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(2, 997, fail_rank=1)
    assert res[1][0] == "error" and "planted failure" in res[1][1]
    assert res[0][0] == "error"  # the survivor's all-reduce ended with an error
