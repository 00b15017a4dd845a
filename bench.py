"""Benchmark of the DeLS draft-scoring hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

One JSON line (rank 0).  A *step* is one pass of the hot path over one batch:
rank projection + fused long-logit / low-rank / prior scoring + argmax (+ for N > 1 the
NCCL all-reduce(MAX) of the packed per-row keys and their decode).

Workloads (seeded synthetic inputs, see dels_b200.workloads):
  * N = 1 default: Qwen3-8B shape bf16, 32 x 16 = 512 rows, H = 4096, r = 256,
    V = 151936 (the configuration the headline metric is quoted on);
  * N > 1 default: the vocab-sharded large batch, 16384 rows, each rank owning a
    contiguous vocabulary slice of W / Vr / prior (strong scaling: total work fixed);
  * ``--workload cfg1|cfg2|cfg3|cfg4|cfg5`` selects any of the five explicitly;
  * ``--workload runner|domino|markov`` times the drop-in rollout runners (DeLSGraphRunner,
    DraftCorrectionGraphRunner, MarkovDeLSGraphRunner) call by call, batch ``--runner-batch``.

``value`` is device-timed (CUDA events, max over ranks) with inputs resident in HBM;
``e2e`` is the same metric through the public API with the step's input rows copied
from pinned host memory and the token ids copied back, inside the timed region.
``roofline`` is the dominant kernel (the fused scorer) timed alone on its stream.
``--impl reference`` times the reference formula (a torch restatement of
code/kernel/dels.py:447-456 with the long logits of code/dflash.py:468) on the host
cores instead.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "dels-spec_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "fused draft-score argmax rows/s @Qwen3-8B shape; % of TC/HBM roofline"
L2_BYTES = 126 * 1024 * 1024


def peaks() -> tuple[float, float, str]:
    """(bf16 TFLOP/s burst, HBM GB/s, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def peaks_sustained() -> float:
    """bf16 TFLOP/s sustained under the power cap (seconds-long GEMM loop)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"])
    return 1400.0


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: torch.device):
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            self.index = str(dev.index or 0)
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"dels_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def ready(self, timeout_s: float = 5.0) -> None:
        """Wait (host only, bounded) until nvidia-smi has written its first sample: its start-up
        can outlast a short load phase, which would leave the record empty."""
        t0 = time.perf_counter()
        while self.proc is not None and time.perf_counter() - t0 < timeout_s:
            try:
                if any(len(line.split(",")) >= 9 for line in self.path.read_text().splitlines()):
                    return
            except OSError:
                pass
            if self.proc.poll() is not None:
                return
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [x for x in sm if x > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- dist
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def default_workload(world: int) -> str:
    """cfg2 (512 rows, the headline) for a plain single-process run; the vocabulary-sharded
    cfg5 (16384 rows) whenever the process was started by torch.distributed.run, N = 1
    included, so that every point of a 1/2/4/8-GPU scaling run times the same workload."""
    under_torchrun = "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ
    return "cfg5" if (world > 1 or under_torchrun) else "cfg2"


def dense_workload_for(wname: str, dev, v_slice=None):
    """The seeded dense workload (cfg1 / cfg2 / cfg5), optionally one vocabulary slice."""
    from dels_b200 import workloads

    if v_slice is None:
        return {"cfg1": workloads.cfg1, "cfg2": workloads.cfg2, "cfg5": workloads.cfg5}[wname](device=dev)
    base = {"cfg2": dict(rows=512, alpha=workloads.linspace(0.5, 0.1, 16), beta=workloads.linspace(0.3, 0.0, 16),
                         seed=1),
            "cfg5": dict(rows=16384, alpha=[0.3], beta=[0.3], seed=4)}[wname]
    name = {"cfg2": "cfg2_qwen3_8b_bf16_b32x16", "cfg5": "cfg5_vocab_sharded_16384"}[wname]
    return workloads.dense_workload(name, H=4096, r=256, dtype=torch.bfloat16, device=dev, v_slice=v_slice, **base)


# The config dict of each workload, built by one function that both arms call, so the
# reference arm's line carries exactly our arm's config.
def dense_config(name: str, rows: int, H: int, r: int, V: int, world: int, sharded: bool) -> dict:
    from dels_b200 import workloads

    v0, v1 = workloads.shard_range(V, world, 0) if sharded else (0, V)
    return {"workload": name, "rows": rows, "H": H, "r": r, "V": V, "vocab_per_rank": v1 - v0,
            "parallelism": f"vocab-shard x{world}" if sharded else "single",
            "l2": "W alone is larger than L2 (streamed from HBM every step)"}


def ragged_config(name: str, n_seq: int, P: int, accepted: int, H: int, r: int, V: int) -> dict:
    return {"workload": name, "sequences": n_seq, "draft": P, "accepted_rows": accepted, "H": H, "r": r, "V": V,
            "l2": "W alone is larger than L2"}


def rnn_config(name: str, rows: int, H: int, r: int, V: int) -> dict:
    return {"workload": name, "rows": rows, "H": H, "r": r, "V": V, "l2": "W alone is larger than L2"}


def runner_config(inp) -> dict:
    return {"workload": inp.name, "V": inp.V, "E": inp.E, "G": inp.G, "r": inp.r,
            "note": "one step = one runner call (14 scored positions per sequence)"}


def markov_config(inp) -> dict:
    return {"workload": inp.name, "V": inp.V, "r": inp.r,
            "note": "one step = one MarkovDeLSGraphRunner call (14 scored positions per sequence)"}


def domino_config(inp) -> dict:
    return {"workload": inp.name, "V": inp.V, "H": inp.H, "G": inp.G, "M": inp.M, "prefix_tokens": inp.P,
            "note": "one step = one DraftCorrectionGraphRunner call (14 scored positions per sequence)"}


class PipelinedE2E:
    """Serving-style end-to-end loop through the public API.

    Every step copies its input rows host -> device (pinned memory) on an H2D stream,
    scores them on the compute stream once they have landed, and copies the token ids
    back on a D2H stream.  Two device input / output slots let the copy of step i+1
    overlap the scoring of step i, as a serving loop would; all copies stay inside the
    timed region (``drain`` makes the compute stream wait for the last read-back)."""

    def __init__(self, host_in: torch.Tensor, score, rows: int, dev, stream):
        self.host_in = host_in
        self.score = score
        self.stream = stream
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.dev_in = [torch.empty_like(host_in, device=dev) for _ in range(2)]
        self.tokens = [torch.empty(rows, dtype=torch.int64, device=dev) for _ in range(2)]
        self.host_out = [torch.empty(rows, dtype=torch.int64).pin_memory() for _ in range(2)]
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.done = [torch.cuda.Event() for _ in range(2)]
        self.read = [torch.cuda.Event() for _ in range(2)]
        for e in self.done + self.read:
            e.record(stream)
        self.i = 0

    def step(self):
        slot = self.i & 1
        self.i += 1
        with torch.cuda.stream(self.h2d):
            self.h2d.wait_event(self.done[slot])  # the slot's previous scoring has consumed it
            self.dev_in[slot].copy_(self.host_in, non_blocking=True)
            self.in_ready[slot].record(self.h2d)
        self.stream.wait_event(self.in_ready[slot])
        self.stream.wait_event(self.read[slot])  # the slot's previous tokens were read back
        self.score(self.dev_in[slot], self.tokens[slot])
        self.done[slot].record(self.stream)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.done[slot])
            self.host_out[slot].copy_(self.tokens[slot], non_blocking=True)
            self.read[slot].record(self.d2h)

    def drain(self):
        self.stream.wait_stream(self.d2h)


class PipelinedE2ESplit:
    """PipelinedE2E for a step made of a rank projection and a scorer (single GPU, bf16).

    The step's kernels form a programmatic-dependent-launch chain (projection,
    finalisation, scorer, next projection, ...); a cross-stream wait or event record
    between two of them makes the second start only after the first has drained.  Here
    every such stream operation sits between the finalisation of step i and its scorer,
    so the scorer of step i still chains into the projection of step i+1:

      compute:  proj(i) fin(i) | record mid(i) | wait in_ready(i+1), read(i-3) | scorer(i)
      h2d:      wait mid(i-1) (scorer(i-2) done: slot free) -> copy input i+1 -> in_ready(i+1)
      d2h:      wait mid(i) (scorer(i-1) done) -> copy tokens of step i-1 -> read(i-1)

    Three input / token slots; every step's input is copied host -> device and every
    step's tokens device -> host inside the timed region (``drain`` reads back the last
    step's tokens and makes the compute stream wait for it)."""

    SLOTS = 3

    def __init__(self, host_in: torch.Tensor, project, score, rows: int, dev, stream):
        n = self.SLOTS
        self.host_in = host_in
        self.project = project
        self.score = score
        self.stream = stream
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.dev_in = [torch.empty_like(host_in, device=dev) for _ in range(n)]
        self.tokens = [torch.empty(rows, dtype=torch.int64, device=dev) for _ in range(n)]
        self.host_out = [torch.empty(rows, dtype=torch.int64).pin_memory() for _ in range(n)]
        self.in_ready = [torch.cuda.Event() for _ in range(n)]
        self.mid = [torch.cuda.Event() for _ in range(n)]
        self.read = [torch.cuda.Event() for _ in range(n)]
        self.last = torch.cuda.Event()
        for e in self.mid + self.read:
            e.record(stream)
        with torch.cuda.stream(self.h2d):
            self.h2d.wait_stream(stream)
            self.dev_in[0].copy_(host_in, non_blocking=True)
            self.in_ready[0].record(self.h2d)
        stream.wait_event(self.in_ready[0])
        self.i = 0

    def step(self):
        n = self.SLOTS
        i = self.i
        self.i += 1
        s, nxt, prev = i % n, (i + 1) % n, (i - 1) % n
        with torch.cuda.stream(self.h2d):
            self.h2d.wait_event(self.mid[prev])  # scorer(i-2) done: slot nxt is free
            self.dev_in[nxt].copy_(self.host_in, non_blocking=True)
            self.in_ready[nxt].record(self.h2d)
        self.project(self.dev_in[s], s)
        self.mid[s].record(self.stream)  # after fin(i): scorer(i-1) has completed
        if i > 0:
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.mid[s])
                self.host_out[prev].copy_(self.tokens[prev], non_blocking=True)
                self.read[prev].record(self.d2h)
        self.stream.wait_event(self.in_ready[nxt])
        self.stream.wait_event(self.read[s])  # tokens slot s of step i-3 was read back
        self.score(self.dev_in[s], s, self.tokens[s])

    def drain(self):
        if self.i == 0:
            return
        prev = (self.i - 1) % self.SLOTS
        self.last.record(self.stream)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.last)
            self.host_out[prev].copy_(self.tokens[prev], non_blocking=True)
        self.stream.wait_stream(self.d2h)


class PipelinedCall:
    """End-to-end loop around a call ``fn(*device_inputs) -> tensor or tuple of tensors``.

    Each step copies its host inputs (pinned) to one of two device slots on an H2D stream
    while the previous call runs, makes the call on the compute stream once they have
    landed, and copies what it returns back to pinned host memory on a D2H stream (the
    returned tensors must not be overwritten by the next call: return clones, or the
    runners' own fresh outputs); ``drain`` makes the compute stream wait for the last
    read-back.  All copies stay inside the timed region."""

    def __init__(self, host_inputs, fn, dev, stream):
        self.host = host_inputs
        self.fn = fn
        self.stream = stream
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.dev_in = [[torch.empty_like(t, device=dev) for t in host_inputs] for _ in range(2)]
        self.host_out = [None, None]
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.done = [torch.cuda.Event() for _ in range(2)]
        for e in self.done:
            e.record(stream)
        self.i = 0

    def step(self):
        slot = self.i & 1
        self.i += 1
        with torch.cuda.stream(self.h2d):
            self.h2d.wait_event(self.done[slot])  # the slot's previous call has consumed it
            for d, h in zip(self.dev_in[slot], self.host):
                d.copy_(h, non_blocking=True)
            self.in_ready[slot].record(self.h2d)
        self.stream.wait_event(self.in_ready[slot])
        outs = self.fn(*self.dev_in[slot])
        outs = [outs] if isinstance(outs, torch.Tensor) else list(outs)
        self.done[slot].record(self.stream)
        if self.host_out[slot] is None:
            self.host_out[slot] = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.done[slot])
            for h, o in zip(self.host_out[slot], outs):
                h.copy_(o, non_blocking=True)
                o.record_stream(self.d2h)

    def drain(self):
        self.stream.wait_stream(self.d2h)


def timed(fn, steps: int, warmup: int, world: int, stream, dev=None, clocks=None, hold_ms: float = 0.0,
          drain=None) -> float:
    """ms for exactly `steps` calls of fn: CUDA events on `stream`, barrier + synchronize on
    both sides.  With `clocks`, the nvidia-smi sampler runs from before a load phase of
    about `hold_ms` (same step count on every rank) until the timed region has ended, so
    the clock record covers the timed region under steady load."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(warmup):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    hold_steps = 0
    if hold_ms > 0:
        est = max_over_ranks(start.elapsed_time(end) / max(warmup, 1), world, dev)
        hold_steps = int(min(5000, max(1, hold_ms / max(est, 1e-3))))
        if clocks is not None:
            clocks.start()
            clocks.ready()
        for _ in range(hold_steps):
            fn()
        torch.cuda.synchronize()
    if drain is not None:
        drain()
    barrier(world)
    start.record(stream)
    for _ in range(steps):
        fn()
    if drain is not None:
        drain()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end)


# ----------------------------------------------------------------------------- CPU reference
def reference_rows_per_s(h, W, w_rank, Vr, prior, alpha_rows, beta_rows, reps: int, rnn=None) -> tuple[float, int]:
    """Time the reference formula (torch on the host) on the given rows; returns rows/s.
    rnn = (w_in, w_s, bias, T): the rank states come from the RNN head's recurrence."""
    from oracle.reference_torch import rnn_rank_states, score_rows

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def once(n):
        state = None if rnn is None else rnn_rank_states(h[:n], *rnn)
        score_rows(h[:n], W, w_rank, Vr, prior, alpha_rows[:n], beta_rows[:n], rank_state=state)

    once(rnn[3] if rnn is not None else 1)  # warm caches
    t0 = time.perf_counter()
    for _ in range(reps):
        once(h.shape[0])
    dt = time.perf_counter() - t0
    return h.shape[0] * reps / dt, torch.get_num_threads()


def ragged_sample(wl, rows: int):
    """cfg3 on the host: acceptance as code/dflash.py:645-651 computes it, then the first
    `rows` accepted rows (draft position j of sequence b for j < accept[b]) with their
    positions' schedules."""
    t = wl.tensors
    draft, target = t["draft"].cpu(), t["target"].cpu()
    P = draft.shape[1]
    accept = (draft == target[:, :P]).to(torch.int64).cumprod(1).sum(1)
    seqs, pos = [], []
    for b in range(draft.shape[0]):
        for j in range(int(accept[b])):
            if len(pos) < rows:
                seqs.append(b)
                pos.append(j)
    h = t["hidden"][torch.tensor(seqs, device=t["hidden"].device), torch.tensor(pos, device=t["hidden"].device)]
    a = torch.tensor(wl.alpha, dtype=torch.float64)[pos]
    b = torch.tensor(wl.beta, dtype=torch.float64)[pos]
    return h.cpu(), t["W"].cpu(), t["w_rank"].cpu(), t["Vr"].cpu(), t["prior"].cpu(), a, b


def rnn_sample(wl, n_seq: int):
    """cfg4 on the host: the rows of the first n_seq sequences and the RNN head's weights."""
    t = wl.tensors
    T = wl.n_pos
    pos = torch.arange(n_seq * T) % T
    a = torch.tensor(wl.alpha, dtype=torch.float64)[pos]
    b = torch.tensor(wl.beta, dtype=torch.float64)[pos]
    rnn = (t["w_in"].cpu(), t["w_s"].cpu(), t["bias"].cpu(), T)
    return (t["x"][: n_seq * T].cpu(), t["W"].cpu(), None, t["Vr"].cpu(), t["prior"].cpu(), a, b), rnn


def cpu_sample(wl, rows: int):
    """The first `rows` rows of a dense workload, moved to the host (bounded CPU sample)."""
    t = wl.tensors
    pos = torch.arange(rows) % wl.n_pos
    a = torch.tensor(wl.alpha, dtype=torch.float64)[pos]
    b = torch.tensor(wl.beta, dtype=torch.float64)[pos]
    h = t["h"][:rows].cpu()
    return h, t["W"].cpu(), t["w_rank"].cpu(), t["Vr"].cpu(), t["prior"].cpu(), a, b


# ----------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, dev):
    from dels_b200 import ops, workloads

    pk_tflops, pk_gbs, pk_src = peaks()
    stream = torch.cuda.current_stream(dev)
    wname = args.workload if args.workload != "auto" else default_workload(world)
    # cfg5 is the vocabulary-sharded configuration at every N (N = 1 included, so the
    # points of a 1 -> 8 curve run one code path); other dense workloads shard when N > 1
    sharded = world > 1 or wname == "cfg5"
    if wname in ("cfg1", "cfg2", "cfg5"):
        from dels_b200.sharded import VocabShardedScorer

        V = workloads.VOCAB
        v0, v1 = workloads.shard_range(V, world, rank) if sharded else (0, V)
        if sharded and wname == "cfg1":
            raise SystemExit("cfg1 (fp32, 16 rows) is single-GPU only")
        wl = dense_workload_for(wname, dev, (v0, v1) if world > 1 else None)
        t = wl.tensors
        rows, H, r = wl.rows, wl.H, wl.r
        Vloc = t["W"].shape[0]
        fp32 = wl.dtype == torch.float32
        need = ops._lib.query("dels_score_f32_workspace_bytes" if fp32 else "dels_score_workspace_bytes",
                              rows, H, r)
        ws = ops.Workspace(need, dev)
        if sharded:
            scorer = VocabShardedScorer(t["W"], t["Vr"], t["prior"], t["w_rank"], t["alpha"], t["beta"], v_begin=v0,
                                        n_pos=wl.n_pos, rows=rows, with_scores=False)
            out = scorer.out
            ws = scorer.ws

            def step(h=t["h"]):
                scorer(h)
        else:
            out = ops.ScoreOut(tokens=torch.empty(rows, dtype=torch.int64, device=dev), scores=None,
                               keys=torch.empty(rows, dtype=torch.int64, device=dev))
            score = ops.draft_score_f32 if fp32 else ops.draft_score_bf16

            def step(h=t["h"]):
                score(h, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=wl.n_pos,
                      out=out, ws=ws)

        # projection + finalisation + scorer (fp32: transpose passes); sharded adds the decode
        launches_per_step = (3 if not fp32 else 2 + (rows + 15) // 16 + 1) + (1 if sharded else 0)
        flops_main = 2.0 * rows * Vloc * (H + r)
        bytes_main = (t["W"].numel() * t["W"].element_size() + t["Vr"].numel() * t["Vr"].element_size()
                      + t["prior"].numel() * 4 + rows * (H + r) * t["h"].element_size() + rows * 8)
        # With vocab sharding every rank needs all rows: each rank copies only its 1/N
        # slice from the host and an NCCL all-gather over NVLink rebuilds the batch, so
        # the box moves each input byte over PCIe once instead of N times.
        gather = world > 1 and rows % world == 0
        rows_in = rows // world if gather else rows
        h_host = t["h"][rank * rows_in:(rank + 1) * rows_in].cpu().pin_memory() if gather else t["h"].cpu().pin_memory()
        h_full = torch.empty_like(t["h"]) if gather else None
        bi, bo = h_host.numel() * h_host.element_size(), rows * 8

        if sharded:
            e2e_outs = [scorer.new_out() for _ in range(2)]
            e2e_ws = [scorer.new_workspace() for _ in range(2)]

            def e2e_score(h_in, tokens, _slot=[0]):
                o, w = e2e_outs[_slot[0]], e2e_ws[_slot[0]]
                _slot[0] ^= 1
                o.tokens = tokens
                if gather:
                    torch.distributed.all_gather_into_tensor(h_full, h_in)
                    h_in = h_full
                scorer(h_in, out=o, ws=w)

            pipe = PipelinedE2E(h_host, e2e_score, rows, dev, stream)
        elif not fp32:
            # projection and scorer as two public calls, so the cross-stream waits sit
            # between them (PipelinedE2ESplit)
            n_sl = PipelinedE2ESplit.SLOTS
            sl_s = [torch.empty(rows, r, dtype=torch.bfloat16, device=dev) for _ in range(n_sl)]
            sl_ws = [ops.Workspace(need, dev) for _ in range(n_sl)]
            sl_out = [ops.ScoreOut(tokens=None, scores=None, keys=torch.empty(rows, dtype=torch.int64, device=dev))
                      for _ in range(n_sl)]

            def e2e_project(h_in, slot):
                ops.rank_project_bf16(h_in, t["w_rank"], t["alpha"], n_pos=wl.n_pos, s_scaled=sl_s[slot],
                                      keys=sl_out[slot].keys, want_state=False, ws=sl_ws[slot])

            def e2e_scorer(h_in, slot, tokens):
                o = sl_out[slot]
                o.tokens = tokens
                ops.fused_argmax_bf16(h_in, t["W"], sl_s[slot], t["Vr"], t["prior"], t["beta"], n_pos=wl.n_pos,
                                      keys_ready=True, out=o, ws=sl_ws[slot])

            pipe = PipelinedE2ESplit(h_host, e2e_project, e2e_scorer, rows, dev, stream)
        else:
            e2e_outs = [ops.ScoreOut(tokens=None, scores=None, keys=torch.empty(rows, dtype=torch.int64, device=dev))
                        for _ in range(2)]
            e2e_ws = [ops.Workspace(need, dev) for _ in range(2)]

            def e2e_score(h_in, tokens, _slot=[0]):
                o, w = e2e_outs[_slot[0]], e2e_ws[_slot[0]]
                _slot[0] ^= 1
                o.tokens = tokens
                score(h_in, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=wl.n_pos,
                      out=o, ws=w)

            pipe = PipelinedE2E(h_host, e2e_score, rows, dev, stream)
        e2e_note = ("per rank: this rank's 1/N row slice (all-gathered over NVLink)" if gather else
                    "per rank: all rows")
        e2e_step = pipe.step

        # roofline: the scorer kernel alone (bf16: tcgen05 fused argmax; fp32: fp32 scorer pass)
        if not fp32:
            _, s_scaled = ops.rank_project_bf16(t["h"], t["w_rank"], t["alpha"], n_pos=wl.n_pos, want_state=False)
            ks = ops.ScoreOut(tokens=torch.empty(rows, dtype=torch.int64, device=dev), scores=None,
                              keys=torch.empty(rows, dtype=torch.int64, device=dev))
            ops.keys_init(ks.keys)
            mws = ops.Workspace(1 << 16, dev)

            # keys reset on every call (a small init kernel chained before the scorer): the
            # scorer's epilogue skips chunks below the row's best key so far, so keys left
            # at the previous launch's result would time a launch with less work
            def main_kernel():
                ops.fused_argmax_bf16(t["h"], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=wl.n_pos,
                                      v_begin=v0, keys_ready=False, out=ks, ws=mws)
        else:
            main_kernel = step
    elif wname == "cfg3":
        return run_ragged(args, rank, world, dev)
    elif wname == "cfg4":
        return run_rnn(args, rank, world, dev)
    elif wname == "runner":
        return run_runner(args, rank, world, dev)
    elif wname == "domino":
        return run_domino(args, rank, world, dev)
    elif wname == "markov":
        return run_markov(args, rank, world, dev)
    else:
        raise SystemExit(f"unknown workload {wname}")

    ops.init(dev)
    clocks = ClockSampler(dev)
    ms = timed(step, args.steps, args.warmup, world, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    ms = max_over_ranks(ms, world, dev)
    # e2e and the scorer-alone timing run under the same sustained load as `value`
    ms_e2e = max_over_ranks(timed(e2e_step, args.steps, args.warmup, world, stream, dev, hold_ms=500.0,
                                  drain=pipe.drain), world, dev)
    ms_main = timed(main_kernel, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0) / args.steps
    ws.check()
    bound = "hbm" if fp32 else "tensor"
    if bound == "tensor":
        achieved = flops_main / (ms_main * 1e-3) / 1e12
        # the scorer is timed after a 0.5 s load phase, at the power-capped clocks of a
        # long run: its denominator is the sustained bf16 peak (burst given beside it)
        peak, unit = peaks_sustained(), "TFLOP/s"
    else:
        achieved = bytes_main / (ms_main * 1e-3) / 1e9
        peak, unit = pk_gbs, "GB/s"
    traffic = None
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get(wname if not sharded else f"{wname}_x{world}")
    total_rows = wl.rows  # every rank scores all rows over its vocabulary slice
    res = {
        "metric": METRIC,
        "value": total_rows * args.steps / (ms * 1e-3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None,
        "dtype": "f32" if fp32 else "bf16",
        "data": "synthetic (seeded, shapes and distributions of the workload)",
        "config": dense_config(wl.name, rows, H, r, workloads.VOCAB, world, sharded),
        "e2e": {"value": total_rows * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo, "note": e2e_note},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{pk_src} ({'sustained' if bound == 'tensor' else 'copy'})",
                     "frac_of_burst_peak": achieved / pk_tflops if bound == "tensor" else None,
                     "kernel_ms": ms_main, "algorithmic": flops_main if bound == "tensor" else bytes_main},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nrows = 16 if fp32 else 32
        h, W, w_rank, Vr, prior, a, b = cpu_sample(wl, nrows)
        rps, cores = reference_rows_per_s(h, W, w_rank, Vr, prior, a, b, reps=2)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port",
                               "sample": f"{nrows} rows of the workload x 2 repetitions, full vocabulary, "
                                         f"{str(wl.dtype).replace('torch.', '')} torch on the host"}
    return res


def run_ragged(args, rank, world, dev):
    from dels_b200 import ops, workloads

    if world > 1:
        raise SystemExit("the ragged workload is single-GPU")
    pk_tflops, _, pk_src = peaks()
    wl = workloads.cfg3(device=dev)
    t = wl.tensors
    stream = torch.cuda.current_stream(dev)
    n_seq, P = t["draft"].shape
    acc = torch.empty(n_seq, dtype=torch.int32, device=dev)
    off = torch.empty(n_seq + 1, dtype=torch.int32, device=dev)
    packed = torch.empty(n_seq * P, wl.H, dtype=torch.bfloat16, device=dev)
    row_pos = torch.zeros(n_seq * P, dtype=torch.int32, device=dev)
    out = ops.ScoreOut(tokens=torch.empty(n_seq * P, dtype=torch.int64, device=dev), scores=None,
                       keys=torch.empty(n_seq * P, dtype=torch.int64, device=dev))
    ws = ops.Workspace(ops._lib.query("dels_score_workspace_bytes", n_seq * P, wl.H, wl.r), dev)

    def step(draft=t["draft"], target=t["target"], hidden=t["hidden"]):
        ops.accept_offsets(draft, target, accept=acc, offsets=off)
        ops.pack_rows(hidden, acc, off, packed=packed, row_pos=row_pos)
        ops.draft_score_bf16(packed, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=P,
                             row_pos=row_pos, rows_dev=off[-1:], out=out, ws=ws)

    ops.init(dev)
    step()
    torch.cuda.synchronize()
    total = int(off[-1])
    clocks = ClockSampler(dev)
    ms = timed(step, args.steps, args.warmup, 1, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    hh = {k: t[k].cpu().pin_memory() for k in ("draft", "target", "hidden")}

    def e2e_call(draft, target, hidden):
        step(draft, target, hidden)
        return out.tokens.clone(), acc.clone()

    pipe = PipelinedCall([hh["draft"], hh["target"], hh["hidden"]], e2e_call, dev, stream)
    ms_e2e = timed(pipe.step, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0, drain=pipe.drain)
    flops = 2.0 * total * wl.V * (wl.H + wl.r)
    _, s_scaled = ops.rank_project_bf16(packed[:total], t["w_rank"], t["alpha"], n_pos=P, row_pos=row_pos[:total],
                                        want_state=False)
    ks = ops.ScoreOut(tokens=torch.empty(total, dtype=torch.int64, device=dev), scores=None,
                      keys=torch.empty(total, dtype=torch.int64, device=dev))
    mws = ops.Workspace(1 << 16, dev)
    main = lambda: ops.fused_argmax_bf16(packed[:total], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=P,  # noqa: E731
                                         row_pos=row_pos[:total], keys_ready=False, out=ks, ws=mws)
    ops.keys_init(ks.keys)
    ms_main = timed(main, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0) / args.steps
    ws.check()
    achieved = flops / (ms_main * 1e-3) / 1e12
    res = {
        "metric": METRIC, "value": total * args.steps / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, shapes and distributions of the workload)",
        "config": ragged_config(wl.name, n_seq, P, total, wl.H, wl.r, wl.V),
        "e2e": {"value": total * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": sum(v.numel() * v.element_size() for v in hh.values()),
                "d2h_bytes_per_step": n_seq * P * 8 + n_seq * 4},
        "gpu_launches": 5 * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks_sustained(), "unit": "TFLOP/s",
                     "frac": achieved / peaks_sustained(), "traffic": None, "peak_source": f"{pk_src} (sustained)",
                     "frac_of_burst_peak": achieved / pk_tflops, "kernel_ms": ms_main},
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        nrows = 24
        rps, cores = reference_rows_per_s(*ragged_sample(wl, nrows), reps=2)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port",
                               "sample": f"the first {nrows} accepted rows (acceptance computed on the host) x "
                                         f"full vocabulary x 2 repetitions, bf16 torch on the host"}
    return res


def run_rnn(args, rank, world, dev):
    from dels_b200 import ops, workloads

    if world > 1:
        raise SystemExit("the RNN workload is single-GPU")
    pk_tflops, _, pk_src = peaks()
    wl = workloads.cfg4(device=dev)
    t = wl.tensors
    stream = torch.cuda.current_stream(dev)
    rows = wl.rows
    s_scaled = torch.empty(rows, wl.r, dtype=torch.bfloat16, device=dev)
    out = ops.ScoreOut(tokens=torch.empty(rows, dtype=torch.int64, device=dev), scores=None,
                       keys=torch.empty(rows, dtype=torch.int64, device=dev))
    ws = ops.Workspace(ops._lib.query("dels_rnn_workspace_bytes", 512, 16, wl.H, wl.r), dev)
    mws = ops.Workspace(1 << 16, dev)

    def step(x=t["x"]):
        ops.rnn_rank_states(x, t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=512, T=16, s_scaled=s_scaled,
                            keys=out.keys, ws=ws)
        ops.fused_argmax_bf16(x, t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=16, keys_ready=True,
                              out=out, ws=mws)

    ops.init(dev)
    clocks = ClockSampler(dev)
    ms = timed(step, args.steps, args.warmup, 1, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    x_host = t["x"].cpu().pin_memory()

    def e2e_call(x):
        step(x)
        return out.tokens.clone()

    pipe = PipelinedCall([x_host], e2e_call, dev, stream)
    ms_e2e = timed(pipe.step, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0, drain=pipe.drain)
    ms_main = timed(lambda: ops.fused_argmax_bf16(t["x"], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=16,
                                                  keys_ready=False, out=out, ws=mws),
                    args.steps, args.warmup, 1, stream, dev, hold_ms=500.0) / args.steps
    ws.check()
    flops = 2.0 * rows * wl.V * (wl.H + wl.r)
    achieved = flops / (ms_main * 1e-3) / 1e12
    res = {
        "metric": METRIC, "value": rows * args.steps / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, shapes and distributions of the workload)",
        "config": rnn_config(wl.name, rows, wl.H, wl.r, wl.V),
        "e2e": {"value": rows * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": rows * 8},
        "gpu_launches": 3 * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks_sustained(), "unit": "TFLOP/s",
                     "frac": achieved / peaks_sustained(), "traffic": None, "peak_source": f"{pk_src} (sustained)",
                     "frac_of_burst_peak": achieved / pk_tflops, "kernel_ms": ms_main},
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        sample_t, rnn = rnn_sample(wl, 2)
        rps, cores = reference_rows_per_s(*sample_t, reps=2, rnn=rnn)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port",
                               "sample": "2 sequences x 16 positions through the RNN head x full vocabulary x 2 "
                                         "repetitions, bf16 torch on the host"}
    return res


def runner_launches(runner, steps: int) -> int:
    """Kernels of libdels_b200.so one DeLSGraphRunner call launches (its graph replay)."""
    lm = 1 if hasattr(runner, "_lm_ws") else 0  # the long-logit GEMM of the materialising runner
    if runner._overlap:  # gates + rank GEMV, scorer (with the next step's W_hh h), keys decode
        return lm + 2 * steps + 1
    if runner._split_gru:  # gates, rank GEMV, scorer (with the next step's W_hh h); keys decode
        return lm + 3 * steps + (1 if runner._keys_only else 0)
    dec = 1 if getattr(runner, "_keys_only", False) else 0  # one keys decode per call
    if runner._tc:  # gates; per step rank GEMM + finalisation, scorer; W_hh GEMM + gate finalisation
        return lm + 1 + 3 * steps + (2 if runner._gru_tc_fused else 3) * (steps - 1) + dec
    return lm + 3 * steps + dec  # GRU step, rank GEMV, scorer


def runner_inputs(args, dev):
    """The runner workload's seeded local head (released shapes V = 151936, E = 256,
    G = 1024, r = 256), schedules and call inputs, built with torch alone (shared by both
    arms): base logits [B, 14, V], or with --runner-hidden the target LM head W [V, 4096]
    and the draft hidden states [B, 14, 4096]."""
    import types

    import torch.nn as nn

    import dels as D
    from dels_b200 import workloads

    V, E, G, r, steps, B = workloads.VOCAB, 256, 1024, 256, 14, args.runner_batch
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    stub = type("T", (), {})()
    stub.model = type("M", (), {})()
    stub.model.embed_tokens = nn.Embedding(V, E).to(device=dev, dtype=torch.bfloat16)
    head = D.DeLSLocalHead(target_model=stub, vocab_size=V, embed_dim=E, gru_hidden_dim=G, low_rank_dim=r,
                           lm_head_mode="low_rank", dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        for p, std in ((head.embed_tokens.weight, 0.5), (head.prefix_gru.weight_ih_l0, 0.05),
                       (head.prefix_gru.weight_hh_l0, 0.03), (head.rank_proj.weight, 0.05),
                       (head.low_rank_lm_head.weight, 0.05)):
            p.copy_(torch.randn(p.shape, generator=g, device=dev) * std)
    inp = types.SimpleNamespace(V=V, E=E, G=G, r=r, steps=steps, B=B, H=4096, head=head, W=None, x=None, base=None)
    inp.prior = workloads.zipf_log_prior(V, device=dev).to(torch.bfloat16)
    inp.alpha = workloads.linspace(0.9, 0.3, steps)
    inp.beta = workloads.linspace(0.3, 0.1, steps)
    inp.prefix = torch.randint(0, V, (B, 1), generator=g, device=dev)
    if args.runner_hidden:
        inp.W = (torch.randn(V, inp.H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        inp.x = torch.randn(B, steps, inp.H, generator=g, device=dev).to(torch.bfloat16)
        inp.name = f"runner_hidden_b{B}_steps{steps}"
    else:
        inp.base = (torch.randn(B, steps, V, generator=g, device=dev)).to(torch.bfloat16)
        inp.name = f"runner_b{B}_steps{steps}"
    return inp


def runner_cpu_rate(inp, reps: int = 2) -> tuple[float, int, str]:
    """The reference's torch rollout (oracle/reference_torch.runner_rollout) of the first
    sequence on the host cores; returns (rows/s, threads, sample)."""
    from oracle.reference_torch import runner_rollout

    torch.set_num_threads(os.cpu_count() or 1)
    head = inp.head
    table = torch.nn.functional.linear(head.embed_tokens.weight, head.prefix_gru.weight_ih_l0).cpu()
    base1 = (torch.nn.functional.linear(inp.x[:1], inp.W) if inp.x is not None else inp.base[:1]).cpu()
    cpu_args = (inp.prefix[:1].cpu(), base1, table, head.prefix_gru.weight_hh_l0.detach().cpu(),
                head.rank_proj.weight.detach().cpu(), head.low_rank_lm_head.weight.detach().cpu(), inp.prior.cpu(),
                inp.alpha, inp.beta)
    runner_rollout(*cpu_args)
    t0 = time.perf_counter()
    for _ in range(reps):
        runner_rollout(*cpu_args)
    dt = (time.perf_counter() - t0) / reps
    return inp.steps / dt, torch.get_num_threads(), \
        f"one batch-1 rollout of {inp.steps} steps x {reps} repetitions, bf16 torch on the host"


def reference_gpu_runner(args, kw, ours, prefix, base, stream, dev, module: str = "dels",
                         cls: str = "DeLSGraphRunner") -> dict:
    """The reference's own DeLSGraphRunner (Triton kernels, code/kernel/dels.py:214-478) on
    this GPU, beside ours: same local head, schedules, prior and call inputs.  The
    reference tree is not part of this repository; ``--reference-runner`` names a copy of
    its ``code/`` directory, whose ``kernel/dels.py`` is loaded under a module name of its
    own.  Returns its ms per call (same timing as ours) and how many tokens agree (a
    greedy rollout may part ways after a near-tie of the scores)."""
    import importlib.util

    path = Path(args.reference_runner) / "kernel" / f"{module}.py"
    spec = importlib.util.spec_from_file_location(f"dels_reference_kernel_{module}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ref = getattr(mod, cls)(**kw)
    ms = timed(lambda: ref(prefix, base), args.steps, args.warmup, 1, stream, dev, hold_ms=300.0) / args.steps
    ms_ours = timed(lambda: ours(prefix, base), args.steps, args.warmup, 1, stream, dev, hold_ms=300.0) / args.steps
    t_ref, t_ours = ref(prefix, base), ours(prefix, base)
    torch.cuda.synchronize()
    same = (t_ref == t_ours)
    first_diff = [int(torch.nonzero(~row).min()) if not bool(row.all()) else None for row in same]
    return {"ms_per_call": ms, "ms_per_call_ours_same_run": ms_ours, "speedup": ms / ms_ours,
            "uses_triton": bool(getattr(ref, "_can_triton_fuse", False)),
            "tokens_identical_frac": float(same.float().mean()), "first_differing_step_per_row": first_diff[:8],
            "source": f"the reference's code/kernel/{module}.py, loaded from --reference-runner at run time"}


def run_runner(args, rank, world, dev):
    """The drop-in DeLSGraphRunner (kernel/dels.py) at the released local-head shapes
    (V = 151936, E = 256, G = 1024, r = 256), batch B, 14 suffix steps: one call =
    copy-in of prefix ids and base logits, CUDA-graph replay, clone of the tokens —
    exactly the reference runner's __call__ (code/kernel/dels.py:469-478)."""
    from kernel.dels import DeLSGraphRunner

    if world > 1:
        raise SystemExit("the runner workload is single-GPU")
    inp = runner_inputs(args, dev)
    V, E, G, r, steps, B = inp.V, inp.E, inp.G, inp.r, inp.steps, inp.B
    head, prior, alpha, beta, prefix = inp.head, inp.prior, inp.alpha, inp.beta, inp.prefix
    kw = dict(local_head=head, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha, beta_values=beta,
              baseline_logits=prior, device=dev)
    stream = torch.cuda.current_stream(dev)
    per_step = (r * V + 3 * G * G + r * G + B * V + B * 3 * G) * 2  # Vr, W_hh, W_rank, base row, table rows
    extra = {}
    if args.runner_hidden:
        # DeLSFusedGraphRunner: the call takes the draft hidden states [B, steps, H] and the
        # runner owns the target LM head (Qwen3-8B shape, H = 4096)
        from kernel.dels import DeLSFusedGraphRunner

        H, W, x = inp.H, inp.W, inp.x
        runner = DeLSFusedGraphRunner(target_lm_head_weight=W, **kw)
        if runner._fused:  # W streamed by every step's scorer
            bytes_call = steps * (per_step - B * V * 2 + V * H * 2 + B * H * 2)
        else:  # one GEMM over all rows writes the logits, the steps read them back
            bytes_call = V * H * 2 + B * steps * H * 2 + B * steps * V * 2 + steps * per_step
        # the reference's flow for comparison: lm_head by torch (cuBLAS), slice copy into
        # the base-logit runner (code/dflash.py:468, :482-485)
        plain = DeLSGraphRunner(**kw)
        unfused = lambda: plain(prefix, torch.nn.functional.linear(x, W))  # noqa: E731
        ms_unfused = timed(unfused, args.steps, args.warmup, 1, stream, dev, hold_ms=300.0)
        extra = {"schedule": "fused per-step scorer" if runner._fused else "one long-logit GEMM per call",
                 "ms_per_call_torch_lm_head_then_base_runner": ms_unfused / args.steps}
        del plain
        inputs = [prefix, x]
    else:
        runner = DeLSGraphRunner(**kw)
        bytes_call = steps * per_step + B * steps * V * 2 * 2  # + copy-in of the base logits (read + write)
        inputs = [prefix, inp.base]
    call = lambda: runner(*inputs)  # noqa: E731
    clocks = ClockSampler(dev)
    ms = timed(call, args.steps, args.warmup, 1, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    host = [t.cpu().pin_memory() for t in inputs]
    pipe = PipelinedCall(host, runner, dev, stream)
    ms_e2e = timed(pipe.step, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0, drain=pipe.drain)
    _, pk_gbs, pk_src = peaks()
    achieved = bytes_call / (ms / args.steps * 1e-3) / 1e9
    rows = B * steps
    res = {
        "metric": METRIC, "value": rows * args.steps / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, random-init local head at the released shapes)",
        "config": runner_config(inp),
        "e2e": {"value": rows * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host),
                "d2h_bytes_per_step": B * steps * 8},
        "gpu_launches": runner_launches(runner, steps) * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk_gbs, "unit": "GB/s", "frac": achieved / pk_gbs,
                     "traffic": None, "peak_source": f"{pk_src} (copy)", "algorithmic": bytes_call,
                     "note": "every step reads Vr (77.8 MB) and W_hh from HBM: the 126 MB L2 does not keep "
                             "Vr across steps under any cache policy measured"},
        "clocks": clk,
    }
    if extra:
        res["runner_schedule"] = extra
    if args.reference_runner and not args.runner_hidden:
        res["reference_gpu_runner"] = reference_gpu_runner(args, kw, runner, prefix, inp.base, stream, dev)
    if not args.no_cpu_baseline:
        rps, cores, sample = runner_cpu_rate(inp)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample}
    return res


def markov_inputs(args, dev):
    """The Markov workload's seeded local head (embedding and LM-head factors [V, r], r =
    256 like the low-rank head), schedules and call inputs (previous token ids, base logits
    [B, 14, V]), built with torch alone (shared by both arms)."""
    import types

    import dels as D
    from dels_b200 import workloads

    V, r, steps, B = workloads.VOCAB, 256, 14, args.runner_batch
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    emb = torch.randn(V, r, generator=g, device=dev) * 0.5
    lm = torch.randn(V, r, generator=g, device=dev) * 0.05
    head = D.MarkovDeLSLocalHead(embedding_weight=emb, lm_head_weight=lm, dtype=torch.bfloat16, device=dev)
    inp = types.SimpleNamespace(V=V, r=r, steps=steps, B=B, head=head, name=f"markov_b{B}_steps{steps}")
    inp.prior = workloads.zipf_log_prior(V, device=dev).to(torch.bfloat16)
    inp.alpha = workloads.linspace(0.9, 0.3, steps)
    inp.beta = workloads.linspace(0.3, 0.1, steps)
    inp.prev = torch.randint(0, V, (B, 1), generator=g, device=dev)
    inp.base = torch.randn(B, steps, V, generator=g, device=dev).to(torch.bfloat16)
    return inp


def markov_cpu_rate(inp, reps: int = 2) -> tuple[float, int, str]:
    """The reference Markov runner's torch path (oracle/reference_torch.markov_rollout) for
    the first sequence on the host cores; returns (rows/s, threads, sample)."""
    from oracle.reference_torch import markov_rollout

    torch.set_num_threads(os.cpu_count() or 1)
    cpu_args = (inp.prev[:1].cpu(), inp.base[:1].cpu(), inp.head.embedding_weight.detach().cpu(),
                inp.head.lm_head_weight.detach().cpu(), inp.prior.cpu(), inp.alpha, inp.beta)
    markov_rollout(*cpu_args)
    t0 = time.perf_counter()
    for _ in range(reps):
        markov_rollout(*cpu_args)
    dt = (time.perf_counter() - t0) / reps
    return inp.steps / dt, torch.get_num_threads(), \
        f"one batch-1 rollout of {inp.steps} steps x {reps} repetitions, bf16 torch on the host"


def run_markov(args, rank, world, dev):
    """The drop-in MarkovDeLSGraphRunner (kernel/markov_dels.py) with a rank-256 Markov head
    over V = 151936, batch B, 14 suffix steps: one call = copy-in of the previous token ids
    and base logits, CUDA-graph replay, clone of the tokens (code/kernel/markov_dels.py:303-312)."""
    from kernel.markov_dels import MarkovDeLSGraphRunner

    if world > 1:
        raise SystemExit("the markov workload is single-GPU")
    inp = markov_inputs(args, dev)
    V, r, steps, B = inp.V, inp.r, inp.steps, inp.B
    kw = dict(local_head=inp.head, batch_size=B, steps=steps, vocab_size=V, alpha_values=inp.alpha,
              beta_values=inp.beta, baseline_logits=inp.prior, device=dev)
    runner = MarkovDeLSGraphRunner(**kw)
    stream = torch.cuda.current_stream(dev)
    call = lambda: runner(inp.prev, inp.base)  # noqa: E731
    clocks = ClockSampler(dev)
    ms = timed(call, args.steps, args.warmup, 1, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    host = [t.cpu().pin_memory() for t in (inp.prev, inp.base)]
    pipe = PipelinedCall(host, runner, dev, stream)
    ms_e2e = timed(pipe.step, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0, drain=pipe.drain)
    _, pk_gbs, pk_src = peaks()
    # per step: the LM-head factor (V x r), the step's base-logit rows, the prior (fp32), the
    # embedding rows; per call: the copy-in of the base logits (read + write)
    per_step = r * V * 2 + B * V * 2 + V * 4 + B * r * 2
    bytes_call = steps * per_step + B * steps * V * 2 * 2
    achieved = bytes_call / (ms / args.steps * 1e-3) / 1e9
    rows = B * steps
    res = {
        "metric": METRIC, "value": rows * args.steps / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, random-init Markov head at the low-rank head's rank)",
        "config": markov_config(inp),
        "e2e": {"value": rows * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host),
                "d2h_bytes_per_step": B * steps * 8},
        "gpu_launches": (2 * steps + 1) * args.steps,  # per step the embedding gather and the scorer; keys decode
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk_gbs, "unit": "GB/s", "frac": achieved / pk_gbs,
                     "traffic": None, "peak_source": f"{pk_src} (copy)", "algorithmic": bytes_call},
        "clocks": clk,
    }
    if args.reference_runner:
        res["reference_gpu_runner"] = reference_gpu_runner(args, kw, runner, inp.prev, inp.base, stream, dev,
                                                           module="markov_dels", cls="MarkovDeLSGraphRunner")
    if not args.no_cpu_baseline:
        rps, cores, sample = markov_cpu_rate(inp)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample}
    return res


def domino_inputs(args, dev):
    """The Domino workload's seeded draft model (GRU and correction MLP, G = M = 1024),
    target embedding and call inputs, built with torch alone (shared by both arms)."""
    import types

    import torch.nn as nn

    from dels_b200 import workloads

    V, H, G, M, steps, P, B = workloads.VOCAB, 4096, 1024, 1024, 14, 2, args.runner_batch
    g = torch.Generator(device=dev)
    g.manual_seed(6)

    class Draft(nn.Module):
        def __init__(self):
            super().__init__()
            self.prefix_gru = nn.GRU(input_size=H, hidden_size=G, num_layers=1, batch_first=True, bias=False)
            self.embed_proj = nn.Sequential(nn.Linear(H + G, M, bias=False), nn.SiLU(), nn.Linear(M, V, bias=False))

    draft = Draft().to(device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in draft.parameters():
            p.copy_(torch.randn(p.shape, generator=g, device=dev) * 0.02)
    stub = type("T", (), {})()
    stub.model = type("M", (), {})()
    stub.model.embed_tokens = nn.Embedding(V, H).to(device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        stub.model.embed_tokens.weight.copy_(torch.randn(V, H, generator=g, device=dev) * 0.02)
    inp = types.SimpleNamespace(V=V, H=H, G=G, M=M, steps=steps, P=P, B=B, alpha=1.0, draft=draft, target=stub,
                                name=f"domino_b{B}_steps{steps}")
    inp.hiddens = torch.randn(B, steps, H, generator=g, device=dev).to(torch.bfloat16)
    inp.base = torch.randn(B, steps, V, generator=g, device=dev).to(torch.bfloat16)
    inp.prefix = torch.randint(0, V, (B, P), generator=g, device=dev)
    return inp


def domino_cpu_rate(inp, reps: int = 2) -> tuple[float, int, str]:
    """The reference runner's torch path (oracle/reference_torch.domino_rollout) for the
    first sequence on the host cores; returns (rows/s, threads, sample)."""
    from oracle.reference_torch import domino_rollout

    torch.set_num_threads(os.cpu_count() or 1)
    cpu = lambda t: t.detach().cpu()  # noqa: E731
    draft, H = inp.draft, inp.H
    w1 = cpu(draft.embed_proj[0].weight)
    table = torch.nn.functional.linear(inp.target.model.embed_tokens.weight, draft.prefix_gru.weight_ih_l0).cpu()
    cpu_args = (inp.prefix[:1].cpu(), inp.hiddens[:1].cpu(), inp.base[:1].cpu(), table,
                cpu(draft.prefix_gru.weight_hh_l0), w1[:, :H].contiguous(), w1[:, H:].contiguous(),
                cpu(draft.embed_proj[2].weight), inp.alpha)
    domino_rollout(*cpu_args)
    t0 = time.perf_counter()
    for _ in range(reps):
        domino_rollout(*cpu_args)
    dt = (time.perf_counter() - t0) / reps
    return inp.steps / dt, torch.get_num_threads(), \
        f"one batch-1 rollout of {inp.steps} steps x {reps} repetitions, bf16 torch on the host"


def run_domino(args, rank, world, dev):
    """The drop-in Domino DraftCorrectionGraphRunner (kernel/domino.py) at Qwen3-8B target
    shapes (V = 151936, H = 4096) with GRU and correction-MLP widths G = M = 1024 (the
    reference fixes no released width), batch B, 14 suffix steps, 2 prefix tokens: one call
    = copy-in of prefix ids, draft hiddens and base logits, graph replay, clone of the tokens
    (code/kernel/domino.py:499-520)."""
    from kernel.domino import DraftCorrectionGraphRunner

    if world > 1:
        raise SystemExit("the domino workload is single-GPU")
    inp = domino_inputs(args, dev)
    V, H, G, M, steps, P, B, alpha = inp.V, inp.H, inp.G, inp.M, inp.steps, inp.P, inp.B, inp.alpha
    draft, stub, hiddens, base, prefix = inp.draft, inp.target, inp.hiddens, inp.base, inp.prefix
    runner = DraftCorrectionGraphRunner(draft_model=draft, target_model=stub, batch_size=B, steps=steps,
                                        hidden_dim=H, gru_hidden_dim=G, vocab_size=V, prefix_token_count=P,
                                        device=dev, guidance_alpha=alpha)
    stream = torch.cuda.current_stream(dev)
    call = lambda: runner(prefix, hiddens, base)  # noqa: E731
    clocks = ClockSampler(dev)
    ms = timed(call, args.steps, args.warmup, 1, stream, dev, clocks, hold_ms=500.0)
    clk = clocks.stop()
    host = [t.cpu().pin_memory() for t in (prefix, hiddens, base)]
    pipe = PipelinedCall(host, runner, dev, stream)
    ms_e2e = timed(pipe.step, args.steps, args.warmup, 1, stream, dev, hold_ms=500.0, drain=pipe.drain)
    _, pk_gbs, pk_src = peaks()
    # per step: fc2 [V, M], W_s [M, G], W_hh [3G, G], base row, table rows; per call: W_z, hiddens,
    # the prefix GRU steps and the copy-in of the base logits (read + write)
    per_step = (V * M + M * G + 3 * G * G + B * V + B * 3 * G) * 2
    bytes_call = steps * per_step + (M * H + B * steps * H + P * (3 * G * G + B * 3 * G)) * 2 + B * steps * V * 4
    achieved = bytes_call / (ms / args.steps * 1e-3) / 1e9
    rows = B * steps
    res = {
        "metric": METRIC, "value": rows * args.steps / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, random-init Domino head; G = M = 1024 assumed)",
        "config": domino_config(inp),
        "e2e": {"value": rows * args.steps / (ms_e2e * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host),
                "d2h_bytes_per_step": B * steps * 8},
        # z GEMM + finalisation, the prefix GRU steps, per step the correction layer and the
        # scorer, and a GRU update (or its gates alone) between steps unless the gates are fused
        # (then one keys decode per call)
        "gpu_launches": (2 + P + 2 * steps + (0 if runner._overlap else steps - 1)
                         + (1 if runner._keys_only else 0)) * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk_gbs, "unit": "GB/s", "frac": achieved / pk_gbs,
                     "traffic": None, "peak_source": f"{pk_src} (copy)", "algorithmic": bytes_call},
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        rps, cores, sample = domino_cpu_rate(inp)
        res["cpu_baseline"] = {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample}
    return res


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, dev, world: int = 1):
    """The reference's CPU formula on the host cores, same workload / metric / unit / config
    as our arm at the same N (rank 0 alone runs it).  Each step is a bounded sample: a few
    dozen rows of the dense workloads (cfg3: accepted rows after the acceptance step; cfg4:
    whole sequences through the RNN head), or one batch-1 rollout for the runners."""
    from dels_b200 import workloads

    wname = args.workload if args.workload != "auto" else default_workload(world)
    gdev = dev if torch.cuda.is_available() else torch.device("cpu")
    if wname in ("runner", "domino", "markov"):
        inputs = {"runner": runner_inputs, "domino": domino_inputs, "markov": markov_inputs}[wname]
        rate = {"runner": runner_cpu_rate, "domino": domino_cpu_rate, "markov": markov_cpu_rate}[wname]
        inp = inputs(args, gdev)
        config = {"runner": runner_config, "domino": domino_config, "markov": markov_config}[wname](inp)
        rates, cores, sample = [], 0, ""
        for i in range(args.warmup + args.steps):
            rps, cores, sample = rate(inp, reps=1)
            if i >= args.warmup:
                rates.append(rps)
        nrows, dtype = inp.steps, "bf16"
    else:
        gen = {"cfg1": workloads.cfg1, "cfg2": workloads.cfg2, "cfg3": workloads.cfg3, "cfg4": workloads.cfg4,
               "cfg5": workloads.cfg5}[wname]
        wl = gen(device=gdev)
        nrows = 16 if wl.dtype == torch.float32 else 24
        rnn = None
        if wname == "cfg3":
            sample_t = ragged_sample(wl, nrows)
            sample = f"the first {nrows} accepted rows x full vocabulary per step, torch on the host"
            draft, target = wl.tensors["draft"].cpu(), wl.tensors["target"].cpu()
            n_seq, P = draft.shape
            accepted = int((draft == target[:, :P]).to(torch.int64).cumprod(1).sum())
            config = ragged_config(wl.name, n_seq, P, accepted, wl.H, wl.r, wl.V)
        elif wname == "cfg4":
            sample_t, rnn = rnn_sample(wl, 2)
            nrows = sample_t[0].shape[0]
            sample = "2 sequences x 16 positions through the RNN head x full vocabulary per step, torch on the host"
            config = rnn_config(wl.name, wl.rows, wl.H, wl.r, wl.V)
        else:
            sample_t = cpu_sample(wl, nrows)
            sample = f"{nrows} rows x full vocabulary per step, torch on the host"
            config = dense_config(wl.name, wl.rows, wl.H, wl.r, wl.V, world, world > 1 or wname == "cfg5")
        sample += f" (rank 0's host cores, {world} rank(s) launched)"
        dtype = "f32" if wl.dtype == torch.float32 else "bf16"
        del wl
        torch.cuda.empty_cache() if torch.cuda.is_available() else None
        rates, cores = [], 0
        for i in range(args.warmup + args.steps):
            rps, cores = reference_rows_per_s(*sample_t, reps=1, rnn=rnn)
            if i >= args.warmup:
                rates.append(rps)
    rps = len(rates) / sum(1.0 / x for x in rates)
    return {
        "metric": METRIC, "value": rps, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": nrows / rps * 1e3, "higher_is_better": True,
        "scaling": "strong" if (world > 1 or wname == "cfg5") else "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic (seeded)",
        "config": config,
        "impl": "reference",
        "cpu_baseline": {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": rps, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="auto",
                    choices=["auto", "cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "runner", "domino", "markov"])
    ap.add_argument("--runner-batch", type=int, default=1, help="batch of the runner workload")
    ap.add_argument("--runner-hidden", action="store_true",
                    help="runner workload: DeLSFusedGraphRunner fed the draft hidden states")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-runner", default="",
                    help="runner / markov workloads: path to a copy of the reference's code/ directory; its "
                         "Triton DeLSGraphRunner / MarkovDeLSGraphRunner is timed beside ours on the same GPU "
                         "and inputs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
        print(json.dumps(run_reference(args, dev, world)), flush=True)
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        res = run_ours(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
