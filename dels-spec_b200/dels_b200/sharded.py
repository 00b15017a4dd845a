"""Vocab-sharded draft scoring across the GPUs of one box.

Each rank owns a contiguous vocabulary slice [v0, v1) of the target LM head W, the
low-rank head Vr and the prior; the draft hidden rows and the rank-projection weight
are replicated.  Every rank scores all rows over its slice and produces one packed
int64 key per row, key = (ordered score << 32) | (0xFFFFFFFF - global index); the
global argmax (lowest index on ties) is then ONE all-reduce(MAX) of rows x 8 bytes
over NCCL, after which every rank decodes the same token ids.

The reference has no counterpart: it parallelises only over prompts
(code/benchmark.py:563) and gathers results with pickled objects
(code/distributed.py:55-72).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops, workloads


def combine_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """In-place all-reduce(MAX) of packed argmax keys (int64); returns ``keys``."""
    if keys.dtype != torch.int64:
        raise ValueError("packed keys must be int64")
    dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return keys


def decode_keys_host(keys: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(token ids, scores) of packed keys with torch ops (any device)."""
    lo = keys & 0xFFFFFFFF
    idx = 0xFFFFFFFF - lo
    hi = (keys >> 32).to(torch.int32)
    bits = torch.where(hi < 0, hi ^ 0x7FFFFFFF, hi)
    return idx.to(torch.int64), bits.view(torch.float32)


class VocabShardedScorer:
    """Scores rows over this rank's vocabulary slice and combines keys across ranks.

    ``W``, ``Vr`` and ``prior`` are the LOCAL slices; ``v_begin`` is the slice's first
    global token id (see :func:`dels_b200.workloads.shard_range`)."""

    def __init__(self, W, Vr, prior, w_rank, alpha, beta, *, v_begin: int, n_pos: int, rows: int,
                 activation: str = "identity", group=None):
        self.W, self.Vr, self.prior, self.w_rank = W, Vr, prior, w_rank
        self.alpha, self.beta = alpha, beta
        self.v_begin, self.n_pos, self.rows = int(v_begin), int(n_pos), int(rows)
        self.activation = activation
        self.group = group
        dev = W.device
        self.out = ops.ScoreOut(tokens=torch.empty(rows, dtype=torch.int64, device=dev),
                                scores=torch.empty(rows, dtype=torch.float32, device=dev),
                                keys=torch.empty(rows, dtype=torch.int64, device=dev))
        H, r = w_rank.shape[1], w_rank.shape[0]
        self.ws = ops.Workspace(ops._lib.query("dels_score_workspace_bytes", rows, H, r), dev)

    def __call__(self, h: torch.Tensor) -> ops.ScoreOut:
        ops.draft_score_bf16(h, self.W, self.w_rank, self.Vr, self.prior, self.alpha, self.beta, n_pos=self.n_pos,
                             v_begin=self.v_begin, activation=self.activation, keys_only=True, out=self.out,
                             ws=self.ws)
        combine_keys(self.out.keys, self.group)
        ops.keys_decode(self.out.keys, tokens=self.out.tokens, scores=self.out.scores)
        return self.out


__all__ = ["combine_keys", "decode_keys_host", "VocabShardedScorer", "workloads"]
