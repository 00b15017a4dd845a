"""One rank of the vocabulary-sharded NCCL check (launched by torch.distributed.run from
tests/test_gpu_sharded_nccl.py; not a test module itself).

Every rank builds the full-size vocabulary-sharded workload (16384 rows, H = 4096,
r = 256, V = 151936, seed 4) restricted to its contiguous vocabulary slice and scores
it with VocabShardedScorer: the tcgen05 scorer writes global-index keys, one NCCL
all-reduce(MAX) combines them, every rank decodes.  A second pass runs the bench's
end-to-end form: each rank holds only its 1/N slice of the hidden rows and an NCCL
all-gather rebuilds the batch before scoring.  Rank 0 then scores the whole vocabulary
on its own GPU with the unsharded entry point and writes a JSON verdict: the sharded
tokens and scores must equal the single-GPU ones bit for bit (every score is computed
with the same arithmetic wherever its vocabulary tile sits, and the maximum of int64
keys is exact).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for _p in (str(ROOT), str(ROOT / "dels-spec_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--rows", type=int, default=16384)
    args = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from dels_b200 import ops, workloads
        from dels_b200.sharded import VocabShardedScorer

        ops.init(dev)
        V = workloads.VOCAB
        v0, v1 = workloads.shard_range(V, world, rank)
        wl = workloads.cfg5(device=dev, v_slice=(v0, v1), rows=args.rows)
        t = wl.tensors
        scorer = VocabShardedScorer(t["W"], t["Vr"], t["prior"], t["w_rank"], t["alpha"], t["beta"], v_begin=v0,
                                    n_pos=wl.n_pos, rows=wl.rows)
        res = scorer(t["h"])
        tok, sc = res.tokens.clone(), res.scores.clone()
        # end-to-end form: this rank's row slice, all-gathered over NVLink
        per = wl.rows // world
        h_full = torch.empty_like(t["h"])
        dist.all_gather_into_tensor(h_full, t["h"][rank * per:(rank + 1) * per].contiguous())
        res2 = scorer(h_full, out=scorer.new_out(), ws=scorer.new_workspace())
        torch.cuda.synchronize()
        scorer.ws.check()
        verdict = {"world": world, "rank": rank, "vocab_slice": [v0, v1]}
        if rank == 0:
            full = workloads.cfg5(device=dev, rows=args.rows)
            ft = full.tensors
            ref = ops.draft_score_bf16(ft["h"], ft["W"], ft["w_rank"], ft["Vr"], ft["prior"], ft["alpha"],
                                       ft["beta"], n_pos=full.n_pos, with_scores=True)
            torch.cuda.synchronize()
            verdict.update(
                rows=wl.rows,
                tokens_equal=bool(torch.equal(tok, ref.tokens)),
                scores_equal=bool(torch.equal(sc, ref.scores)),
                gathered_tokens_equal=bool(torch.equal(res2.tokens, ref.tokens)),
                mismatched_rows=int((tok != ref.tokens).sum().item()),
            )
            Path(args.out).write_text(json.dumps(verdict))
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
