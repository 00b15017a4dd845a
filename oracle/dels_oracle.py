"""CPU oracle for the DeLS draft-scoring hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's algorithm for the path the CUDA library
implements.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker; nothing in ``dels-spec_b200/`` imports it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Python code
(``dels.py``, ``kernel/dels.py``, ``kernel/markov_dels.py``, ``dflash.sample``) on seeded
inputs and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every function below against those fixtures.

Numerics conventions (shared with the CUDA kernels):
  * bf16 values are carried as float32 holding exactly-representable values;
    :func:`bf16_round` is round-to-nearest-even.
  * Contractions accumulate in float64 here (the kernels accumulate in fp32), so the
    oracle is the "exact" score against which the fp32 accumulation is judged.
  * argmax returns the lowest index among equal maxima and treats NaN as the largest
    value — torch.argmax's rule (code/kernel/dels.py:456; strict '>' at :134).
"""

from __future__ import annotations

from typing import Iterable, Sequence

import numpy as np

# ----------------------------------------------------------------------------- bf16


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.float32(np.nan)
    return out.reshape(a.shape)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_to_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ----------------------------------------------------------------------------- schedules / prior


def parse_scalar_schedule(values, steps: int, *, name: str) -> list[float]:
    """Scalar or comma-separated per-position schedule (code/dels.py:93-112)."""
    if isinstance(values, str):
        parsed = [float(p.strip()) for p in values.split(",") if p.strip()]
    elif isinstance(values, (float, int)):
        parsed = [float(values)]
    else:
        parsed = [float(v) for v in values]
    if not parsed:
        raise ValueError(f"{name} schedule cannot be empty.")
    if len(parsed) == 1:
        parsed = parsed * steps
    if len(parsed) != steps:
        raise ValueError(f"{name} schedule length must be 1 or {steps}, got {len(parsed)}.")
    return parsed


def log_unigram_prior(counts: np.ndarray, vocab_size: int, smoothing: float = 1.0) -> np.ndarray:
    """log((c + s) / sum(c + s)) in float64 (code/dels.py:66-88).

    Counts shorter than the vocabulary are zero-padded (:72-75); with smoothing 0 the
    zero-count entries take the smallest finite log-probability (:77-85)."""
    if smoothing < 0:
        raise ValueError("smoothing must be non-negative.")
    c = np.asarray(counts, dtype=np.float64).reshape(-1)
    if c.size > vocab_size:
        raise ValueError(f"Unigram baseline vocab size {c.size} exceeds runtime vocab size {vocab_size}.")
    if c.size < vocab_size:
        c = np.concatenate([c, np.zeros(vocab_size - c.size)])
    if smoothing == 0.0:
        nz = c > 0
        if not nz.any():
            raise ValueError("Unigram baseline has no positive counts.")
        out = np.full_like(c, -np.inf)
        out[nz] = np.log(c[nz]) - np.log(c.sum())
        out[~nz] = out[nz].min()
        return out
    sm = c + float(smoothing)
    return np.log(sm) - np.log(sm.sum())


def zipf_log_prior(vocab_size: int, s: float = 1.1) -> np.ndarray:
    """Synthetic log-unigram prior: token v has Zipf weight (v + 1)^-s, normalised, logged."""
    w = np.arange(1, vocab_size + 1, dtype=np.float64) ** (-float(s))
    return np.log(w / w.sum())


# ----------------------------------------------------------------------------- argmax / keys


def argmax_first(scores: np.ndarray) -> np.ndarray:
    """Row-wise argmax, lowest index on ties, NaN wins (torch.argmax semantics)."""
    s = np.asarray(scores)
    nan = np.isnan(s)
    idx = np.argmax(np.where(nan, -np.inf, s), axis=-1)
    has_nan = nan.any(axis=-1)
    if np.any(has_nan):
        idx = np.where(has_nan, np.argmax(nan, axis=-1), idx)
    return idx.astype(np.int64)


def top2_gap(scores: np.ndarray) -> np.ndarray:
    """best - second best per row (0 when the maximum is tied)."""
    s = np.asarray(scores, dtype=np.float64)
    part = np.partition(s, -2, axis=-1)
    return part[..., -1] - part[..., -2]


def ordered_i32(x: np.ndarray) -> np.ndarray:
    """float32 -> int32 whose signed order is the float order (NaN largest, -0 == +0)."""
    f = np.asarray(x, dtype=np.float32).copy()
    f[f == 0] = 0.0
    i = f.view(np.int32).astype(np.int64)
    o = np.where(i < 0, i ^ 0x7FFFFFFF, i)
    o = np.where(np.isnan(f), 0x7FFFFFFF, o)
    return o.astype(np.int32)


def pack_keys(scores: np.ndarray, index: np.ndarray) -> np.ndarray:
    """Packed int64 argmax keys: (ordered score << 32) | (0xFFFFFFFF - index)."""
    hi = ordered_i32(scores).astype(np.int64)
    lo = (np.int64(0xFFFFFFFF) - np.asarray(index, dtype=np.int64)) & 0xFFFFFFFF
    return (hi << 32) | lo


def key_index(keys: np.ndarray) -> np.ndarray:
    return (np.int64(0xFFFFFFFF) - (np.asarray(keys, dtype=np.int64) & 0xFFFFFFFF)).astype(np.int64)


# ----------------------------------------------------------------------------- scorer


def row_positions(rows: int, n_pos: int, row_pos: np.ndarray | None = None) -> np.ndarray:
    return np.asarray(row_pos, dtype=np.int64) if row_pos is not None else np.arange(rows) % n_pos


def rank_state_bf16(h: np.ndarray, w_rank: np.ndarray, activation: str = "identity") -> np.ndarray:
    """bf16(act(bf16(h . w_rank^T))) — F.linear with bf16 output then F.silu in bf16
    (code/kernel/dels.py:437-439; code/dels.py:334-338)."""
    acc = (np.asarray(h, np.float64) @ np.asarray(w_rank, np.float64).T).astype(np.float32)
    s = bf16_round(acc)
    if activation == "silu":
        s32 = s.astype(np.float32)
        s = bf16_round((s32 / (np.float32(1.0) + np.exp(-s32))).astype(np.float32))
    elif activation != "identity":
        raise ValueError(f"Unsupported DeLS rank_activation={activation!r}.")
    return s


def scores_from_parts(
    long_logits: np.ndarray,
    short_logits: np.ndarray,
    prior: np.ndarray | None,
    alpha_rows: np.ndarray,
    beta_rows: np.ndarray,
) -> np.ndarray:
    """final = long + alpha_p * short - beta_p * prior (code/kernel/dels.py:448-455,
    code/dflash.py:523-527), float64."""
    out = np.asarray(long_logits, np.float64) + np.asarray(alpha_rows, np.float64)[:, None] * np.asarray(
        short_logits, np.float64
    )
    if prior is not None:
        out = out - np.asarray(beta_rows, np.float64)[:, None] * np.asarray(prior, np.float64)[None, :]
    return out


def draft_scores(
    h: np.ndarray,
    W: np.ndarray,
    s: np.ndarray,
    Vr: np.ndarray,
    prior: np.ndarray | None,
    alpha_rows: np.ndarray,
    beta_rows: np.ndarray,
    *,
    v_chunk: int = 16384,
) -> np.ndarray:
    """Full [rows, V] scores h.W^T + alpha_p (s.Vr^T) - beta_p prior in float64.

    The long logits are the target LM head applied to the draft hidden state
    (code/dflash.py:468) and are NOT rounded (the fused path never materialises them)."""
    h64 = np.asarray(h, np.float64)
    s64 = np.asarray(s, np.float64)
    V = W.shape[0]
    out = np.empty((h.shape[0], V), dtype=np.float64)
    for v0 in range(0, V, v_chunk):
        v1 = min(V, v0 + v_chunk)
        long_ = h64 @ np.asarray(W[v0:v1], np.float64).T
        short = s64 @ np.asarray(Vr[v0:v1], np.float64).T
        out[:, v0:v1] = scores_from_parts(long_, short, None if prior is None else prior[v0:v1], alpha_rows, beta_rows)
    return out


def draft_score_bf16(
    h: np.ndarray,
    W: np.ndarray,
    w_rank: np.ndarray,
    Vr: np.ndarray,
    prior: np.ndarray | None,
    alpha: Sequence[float],
    beta: Sequence[float],
    *,
    n_pos: int | None = None,
    row_pos: np.ndarray | None = None,
    activation: str = "identity",
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Tokens, scores [rows, V] and top-2 gaps for the bf16 scorer's semantics:
    bf16 inputs (float32 arrays of bf16 values), rank state rounded to bf16 as the
    reference's F.linear does, everything after in exact arithmetic."""
    alpha = np.asarray(alpha, np.float64)
    beta = np.asarray(beta, np.float64)
    npos = int(n_pos or len(alpha))
    pos = row_positions(h.shape[0], npos, row_pos)
    s = rank_state_bf16(h, w_rank, activation)
    sc = draft_scores(h, W, s, Vr, prior, alpha[pos], beta[pos])
    return argmax_first(sc), sc, top2_gap(sc)


def draft_score_f32(
    h: np.ndarray,
    W: np.ndarray,
    w_rank: np.ndarray,
    Vr: np.ndarray,
    prior: np.ndarray | None,
    alpha: Sequence[float],
    beta: Sequence[float],
    *,
    n_pos: int | None = None,
    row_pos: np.ndarray | None = None,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """fp32 semantics: s = h . w_rank^T kept unrounded."""
    alpha = np.asarray(alpha, np.float64)
    beta = np.asarray(beta, np.float64)
    npos = int(n_pos or len(alpha))
    pos = row_positions(h.shape[0], npos, row_pos)
    s = np.asarray(h, np.float64) @ np.asarray(w_rank, np.float64).T
    sc = draft_scores(h, W, s, Vr, prior, alpha[pos], beta[pos])
    return argmax_first(sc), sc, top2_gap(sc)


def base_scores(
    base: np.ndarray, s: np.ndarray, Vr: np.ndarray, prior: np.ndarray | None, alpha_rows, beta_rows
) -> np.ndarray:
    """Runner step scores: base + alpha_p (s.Vr^T) - beta_p prior (code/kernel/dels.py:70-90)."""
    short = np.asarray(s, np.float64) @ np.asarray(Vr, np.float64).T
    return scores_from_parts(base, short, prior, alpha_rows, beta_rows)


# ----------------------------------------------------------------------------- acceptance


def accept_lengths(draft: np.ndarray, target: np.ndarray) -> np.ndarray:
    """(draft == target[:, :P]).cumprod(1).sum(1) — code/dflash.py:645-651, where
    verify_ids[:, 1:] are the draft tokens and posterior[:, :-1] the target tokens."""
    d = np.asarray(draft)
    t = np.asarray(target)[:, : d.shape[1]]
    return np.cumprod(d == t, axis=1).sum(axis=1).astype(np.int32)


def accept_offsets(draft: np.ndarray, target: np.ndarray, commit_extra: int = 0) -> tuple[np.ndarray, np.ndarray]:
    acc = accept_lengths(draft, target)
    off = np.zeros(acc.shape[0] + 1, dtype=np.int64)
    np.cumsum(acc.astype(np.int64) + commit_extra, out=off[1:])
    return acc, off.astype(np.int32)


def pack_rows(hidden: np.ndarray, accept: np.ndarray, offsets: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """packed[offsets[b] + j] = hidden[b, j] for j < accept[b]; row positions j."""
    n_seq, P, H = hidden.shape
    total = int(offsets[-1])
    packed = np.zeros((total, H), dtype=hidden.dtype)
    pos = np.zeros(total, dtype=np.int32)
    for b in range(n_seq):
        a = int(accept[b])
        o = int(offsets[b])
        packed[o : o + a] = hidden[b, :a]
        pos[o : o + a] = np.arange(a)
    return packed, pos


# ----------------------------------------------------------------------------- RNN local head


def rnn_states(
    x: np.ndarray, w_in: np.ndarray, w_s: np.ndarray, bias: np.ndarray | None, n_seq: int, T: int
) -> np.ndarray:
    """s_t = tanh(W_in x_t + W_s s_{t-1} + b), s_0 = 0, in float64; rows [seq, t]."""
    pre = np.asarray(x, np.float64) @ np.asarray(w_in, np.float64).T
    r = w_in.shape[0]
    pre = pre.reshape(n_seq, T, r)
    ws = np.asarray(w_s, np.float64)
    b = np.zeros(r) if bias is None else np.asarray(bias, np.float64)
    s = np.zeros((n_seq, r))
    out = np.zeros((n_seq, T, r))
    for t in range(T):
        s = np.tanh(pre[:, t] + s @ ws.T + b)
        out[:, t] = s
    return out.reshape(n_seq * T, r)


# ----------------------------------------------------------------------------- GRU runner


def gru_cell(gi: np.ndarray, gh: np.ndarray, h: np.ndarray) -> np.ndarray:
    """Bias-free GRU update from precomputed input / hidden projections
    (code/kernel/dels.py:368-373 and the Triton cell :202-205):
      r = sigmoid(gi_r + gh_r), z = sigmoid(gi_z + gh_z), n = tanh(gi_n + r * gh_n)
      h' = (1 - z) * n + z * h"""
    G = h.shape[-1]
    gi = np.asarray(gi, np.float64)
    gh = np.asarray(gh, np.float64)
    h = np.asarray(h, np.float64)
    r = 1.0 / (1.0 + np.exp(-(gi[..., :G] + gh[..., :G])))
    z = 1.0 / (1.0 + np.exp(-(gi[..., G : 2 * G] + gh[..., G : 2 * G])))
    n = np.tanh(gi[..., 2 * G :] + r * gh[..., 2 * G :])
    return (1.0 - z) * n + z * h


def dels_runner_rollout(
    prefix_ids: np.ndarray,
    base_logits: np.ndarray,
    *,
    embed: np.ndarray,
    w_ih: np.ndarray,
    w_hh: np.ndarray,
    w_rank: np.ndarray,
    Vr: np.ndarray,
    prior: np.ndarray | None,
    alpha: Sequence[float],
    beta: Sequence[float],
    activation: str = "identity",
    bf16: bool = False,
    table: np.ndarray | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """Greedy DeLS suffix rollout of DeLSGraphRunner._forward_impl
    (code/kernel/dels.py:425-467): h = GRU(embed[prefix]); for each step: rank state,
    base + alpha*short - beta*prior, argmax, GRU(embed[token]).

    With ``bf16=True`` the values the reference stores in bf16 tensors are rounded
    (gi table, gh, GRU state, rank state) while the mix is exact — the Triton path's
    semantics (fp32 math on bf16 storage, :47-88 and :164-211).  ``table`` may pass a
    precomputed input table embed . w_ih^T.  Returns tokens [B, steps] and per-step
    top-2 gaps [B, steps]."""
    rnd = bf16_round if bf16 else (lambda a: np.asarray(a, np.float64))
    B = prefix_ids.shape[0]
    steps = base_logits.shape[1]
    G = w_hh.shape[1]
    if table is None:
        table = rnd((np.asarray(embed, np.float64) @ np.asarray(w_ih, np.float64).T).astype(np.float32))
    h = np.zeros((B, G))

    def advance(tok, h):
        gi = np.asarray(table[tok], np.float64)
        gh = np.asarray(rnd((h @ np.asarray(w_hh, np.float64).T).astype(np.float32)), np.float64)
        return np.asarray(rnd(gru_cell(gi, gh, h).astype(np.float32)), np.float64)

    h = advance(np.asarray(prefix_ids).reshape(B), h)
    out = np.zeros((B, steps), dtype=np.int64)
    gaps = np.zeros((B, steps))
    alpha = np.asarray(alpha, np.float64)
    beta = np.asarray(beta, np.float64)
    for step in range(steps):
        acc = (h @ np.asarray(w_rank, np.float64).T).astype(np.float32)
        s = rnd(acc)
        if activation == "silu":
            s32 = np.asarray(s, np.float32)
            s = rnd((s32 / (np.float32(1.0) + np.exp(-s32))).astype(np.float32))
        sc = base_scores(
            base_logits[:, step], s, Vr, prior, np.full(B, alpha[step]), np.full(B, beta[step])
        )
        tok = argmax_first(sc)
        out[:, step] = tok
        gaps[:, step] = top2_gap(sc)
        if step + 1 < steps:
            h = advance(tok, h)
    return out, gaps


def markov_runner_rollout(
    prev_ids: np.ndarray,
    base_logits: np.ndarray,
    *,
    embedding: np.ndarray,
    lm_head: np.ndarray,
    prior: np.ndarray | None,
    alpha: Sequence[float],
    beta: Sequence[float],
) -> tuple[np.ndarray, np.ndarray]:
    """MarkovDeLSGraphRunner._forward_impl (code/kernel/markov_dels.py:285-301): the rank
    state is the embedding row of the previous token."""
    B = prev_ids.shape[0]
    steps = base_logits.shape[1]
    tok = np.asarray(prev_ids).reshape(B)
    out = np.zeros((B, steps), dtype=np.int64)
    gaps = np.zeros((B, steps))
    for step in range(steps):
        s = np.asarray(embedding, np.float64)[tok]
        sc = base_scores(base_logits[:, step], s, lm_head, prior, np.full(B, alpha[step]), np.full(B, beta[step]))
        tok = argmax_first(sc)
        out[:, step] = tok
        gaps[:, step] = top2_gap(sc)
    return out, gaps


def domino_runner_rollout(
    prefix_ids: np.ndarray,
    hiddens: np.ndarray,
    base_logits: np.ndarray,
    *,
    embed: np.ndarray,
    w_ih: np.ndarray,
    w_hh: np.ndarray,
    b_ih: np.ndarray | None,
    b_hh: np.ndarray | None,
    w1: np.ndarray,
    b1: np.ndarray | None,
    fc2: np.ndarray,
    b2: np.ndarray | None,
    alpha: float,
    bf16: bool = False,
) -> tuple[np.ndarray, np.ndarray]:
    """Greedy Domino correction rollout of DraftCorrectionGraphRunner._forward_impl
    (code/kernel/domino.py:399-451) with the fused step of :57-139:

      z      = F.linear(hiddens, W_z, b1)                 W_z = w1[:, :H]   (:404-408)
      h      = GRU over the prefix tokens from h = 0       (:410-414)
      per step t:
        s    = F.linear(h, W_s)                            W_s = w1[:, H:]   (:422)
        mid  = SiLU(z_t + s)                               fp32 in the kernel (:92-97)
        logit= alpha * (mid . fc2^T + b2) + base_t         (:104-121)
        tok  = argmax (first index)                        (:123-173)
        h    = GRUCell(table[tok], h), table = F.linear(embed, W_ih, b_ih)  (:436-447)

    With ``bf16=True`` the tensors the reference keeps in bf16 are rounded (z, the
    table, gh = F.linear(h, W_hh, b_hh), the GRU state, s) and the fused step is exact.
    Returns tokens [B, steps] and per-step top-2 gaps [B, steps]."""
    rnd = bf16_round if bf16 else (lambda a: np.asarray(a, np.float64))
    f64 = lambda a: np.asarray(a, np.float64)  # noqa: E731
    B, steps, H = hiddens.shape
    G = w_hh.shape[1]
    z = f64(rnd((f64(hiddens) @ f64(w1)[:, :H].T + (0.0 if b1 is None else f64(b1))).astype(np.float32)))
    w_s = f64(w1)[:, H:]

    def table_rows(tok):  # rows of F.linear(embed, W_ih, b_ih), only those gathered
        gi = f64(embed)[np.asarray(tok)] @ f64(w_ih).T + (0.0 if b_ih is None else f64(b_ih))
        return f64(rnd(gi.astype(np.float32)))

    def advance(tok, h):
        gh = f64(rnd((h @ f64(w_hh).T + (0.0 if b_hh is None else f64(b_hh))).astype(np.float32)))
        return f64(rnd(gru_cell(table_rows(tok), gh, h).astype(np.float32)))

    h = np.zeros((B, G))
    for p in range(np.asarray(prefix_ids).shape[1]):
        h = advance(np.asarray(prefix_ids)[:, p], h)
    out = np.zeros((B, steps), dtype=np.int64)
    gaps = np.zeros((B, steps))
    for t in range(steps):
        s = f64(rnd((h @ w_s.T).astype(np.float32)))
        pre = z[:, t] + s
        mid = pre / (1.0 + np.exp(-pre))
        logit = mid @ f64(fc2).T
        if b2 is not None:
            logit = logit + f64(b2)[None, :]
        sc = float(alpha) * logit + f64(base_logits[:, t])
        tok = argmax_first(sc)
        out[:, t] = tok
        gaps[:, t] = top2_gap(sc)
        if t + 1 < steps:
            h = advance(tok, h)
    return out, gaps


def iter_seeded(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


__all__: Iterable[str] = [n for n in dir() if not n.startswith("_")]
