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
    global token id (see :func:`dels_b200.workloads.shard_range`).  With one rank (or
    no process group) the combine is skipped and the same scorer serves the whole
    vocabulary, so the 1-GPU point of a scaling curve runs the same code path.

    A call enqueues the scorer, the all-reduce(MAX) and the decode on the current
    stream and returns ``out`` (default: the scorer's own buffers).  Callers that keep
    several calls in flight pass their own ``out`` / ``ws`` per call."""

    def __init__(self, W, Vr, prior, w_rank, alpha, beta, *, v_begin: int, n_pos: int, rows: int,
                 activation: str = "identity", with_scores: bool = True, group=None):
        self.W, self.Vr, self.prior, self.w_rank = W, Vr, prior, w_rank
        self.alpha, self.beta = alpha, beta
        self.v_begin, self.n_pos, self.rows = int(v_begin), int(n_pos), int(rows)
        self.activation = activation
        self.with_scores = bool(with_scores)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.out = self.new_out()
        self.ws = self.new_workspace()

    def workspace_bytes(self) -> int:
        H, r = self.w_rank.shape[1], self.w_rank.shape[0]
        return int(ops._lib.query("dels_score_workspace_bytes", self.rows, H, r))

    def new_workspace(self) -> ops.Workspace:
        return ops.Workspace(self.workspace_bytes(), self.W.device)

    def new_out(self) -> ops.ScoreOut:
        dev = self.W.device
        return ops.ScoreOut(tokens=torch.empty(self.rows, dtype=torch.int64, device=dev),
                            scores=torch.empty(self.rows, dtype=torch.float32, device=dev) if self.with_scores
                            else None,
                            keys=torch.empty(self.rows, dtype=torch.int64, device=dev))

    def __call__(self, h: torch.Tensor, *, out: ops.ScoreOut | None = None,
                 ws: ops.Workspace | None = None) -> ops.ScoreOut:
        out = self.out if out is None else out
        ws = self.ws if ws is None else ws
        ops.draft_score_bf16(h, self.W, self.w_rank, self.Vr, self.prior, self.alpha, self.beta, n_pos=self.n_pos,
                             v_begin=self.v_begin, activation=self.activation, keys_only=True, out=out, ws=ws)
        if self.world > 1:
            combine_keys(out.keys, self.group)
        ops.keys_decode(out.keys, tokens=out.tokens, scores=out.scores, with_scores=self.with_scores)
        return out


__all__ = ["combine_keys", "decode_keys_host", "VocabShardedScorer", "workloads"]
