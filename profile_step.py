"""Profiling entry: a few launches of one kernel of the scoring path, for ncu.

    python profile_step.py --workload cfg2 --kernel scorer --launches 4

The ncu summaries under ``profiles/`` were captured with this script (their commands
name it); ``bench.py`` is the timing entry, this one only launches.

``--kernel scorer`` launches the fused tcgen05 scorer, each call after a small
keys-reset kernel (the scorer's epilogue skips chunks below the row's best key so far,
so every profiled launch starts from empty keys); ``--kernel step`` runs whole draft-scoring steps
(projection + finalisation + scorer); ``--kernel f32`` runs the fp32 scorer step;
``--kernel rnn`` (cfg4) runs the RNN head's rank states alone (input projection +
recurrence) over a 2048-token vocabulary, so that nothing but the head is resident.
All inputs are generated and the rank operand computed before the first profiled
launch, so with ``ncu -k regex:<name> -s <launches-1> -c 1`` the capture is a single
warm launch of that kernel.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "dels-spec_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from dels_b200 import ops, workloads  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="cfg2", choices=["cfg1", "cfg2", "cfg5", "cfg4"])
    ap.add_argument("--kernel", default="scorer", choices=["scorer", "step", "f32", "rnn"])
    ap.add_argument("--launches", type=int, default=4)
    ap.add_argument("--rows", type=int, default=0, help="override the row count (cfg5)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops.init(dev)
    if args.kernel == "rnn" and args.workload != "cfg4":
        raise SystemExit("--kernel rnn needs --workload cfg4")
    if args.workload == "cfg4":
        wl = workloads.cfg4(device=dev, V=2048) if args.kernel == "rnn" else workloads.cfg4(device=dev)
        t = wl.tensors
        s_scaled, _ = ops.rnn_rank_states(t["x"], t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=512, T=16)
        h = t["x"]
    else:
        gen = {"cfg1": workloads.cfg1, "cfg2": workloads.cfg2, "cfg5": workloads.cfg5}[args.workload]
        wl = gen(device=dev, rows=args.rows) if (args.workload == "cfg5" and args.rows) else gen(device=dev)
        t = wl.tensors
        h = t["h"]
        s_scaled = None
        if wl.dtype == torch.bfloat16:
            _, s_scaled = ops.rank_project_bf16(h, t["w_rank"], t["alpha"], n_pos=wl.n_pos, want_state=False)
    out = ops.ScoreOut(tokens=torch.empty(wl.rows, dtype=torch.int64, device=dev), scores=None,
                       keys=torch.empty(wl.rows, dtype=torch.int64, device=dev))
    ops.keys_init(out.keys)
    ws = ops.Workspace(1 << 26, dev)
    torch.cuda.synchronize()
    for _ in range(args.launches):
        if args.kernel == "scorer":
            ops.fused_argmax_bf16(h, t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=wl.n_pos,
                                  keys_ready=False, out=out, ws=ws)
        elif args.kernel == "rnn":
            ops.rnn_rank_states(t["x"], t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=512, T=16,
                                s_scaled=s_scaled, keys=out.keys, ws=ws)
        elif args.kernel == "step":
            ops.draft_score_bf16(h, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=wl.n_pos,
                                 out=out, ws=ws)
        else:
            ops.draft_score_f32(h, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=wl.n_pos,
                                out=out, ws=ws)
    torch.cuda.synchronize()
    ws.check()
    print(f"{args.workload} {args.kernel}: {args.launches} launches ok, rows={wl.rows}")


if __name__ == "__main__":
    main()
