"""The reference's scoring formula as torch ops on the host — TEST / BASELINE ONLY.

Restates, operation for operation and in the reference's own dtype, the CPU path the
reference takes for one draft-scoring step: the long logits of the target LM head
(code/dflash.py:468), the rank state and low-rank logits of the local head
(code/kernel/dels.py:437 and :448), the mix with a Python-float alpha / beta per draft
position (code/kernel/dels.py:449-455, eager twin code/dflash.py:523-527) and
torch.argmax (:456).  ``bench.py`` times it on the host cores as the CPU baseline; it
is never part of the product path.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


@torch.inference_mode()
def score_rows(h, W, w_rank, Vr, prior, alpha_rows, beta_rows, rank_state=None) -> torch.Tensor:
    """Token ids [rows] for rows whose draft positions carry alpha_rows / beta_rows
    (rank_state given: it replaces F.linear(h, w_rank))."""
    long_logits = F.linear(h, W)
    if rank_state is None:
        rank_state = F.linear(h, w_rank)
    short_logits = F.linear(rank_state, Vr)
    prior = None if prior is None else prior.to(long_logits.dtype).view(1, -1)
    out = torch.empty(h.shape[0], dtype=torch.long)
    a = [float(x) for x in alpha_rows]
    b = [float(x) for x in beta_rows]
    for key in sorted(set(zip(a, b))):
        idx = torch.tensor([i for i in range(len(a)) if (a[i], b[i]) == key], dtype=torch.long)
        logits = long_logits[idx] + key[0] * short_logits[idx]
        if prior is not None and key[1] != 0.0:
            logits = logits - key[1] * prior
        out[idx] = torch.argmax(logits, dim=-1)
    return out


@torch.inference_mode()
def runner_rollout(prefix_ids, base_logits, table, w_hh, w_rank, Vr, prior, alpha, beta) -> torch.Tensor:
    """DeLSGraphRunner._forward_impl's torch path (code/kernel/dels.py:425-467 with the
    fallback cell :368-373 and mix :447-456), on the host: GRU over the chosen tokens,
    rank projection, base + alpha * low-rank - beta * prior, argmax, per step."""
    B, steps, _ = base_logits.shape
    G = w_hh.shape[1]
    h = torch.zeros(B, G, dtype=base_logits.dtype)

    def cell(gi, h):
        gh = F.linear(h, w_hh)
        i_r, i_z, i_n = gi.chunk(3, dim=-1)
        h_r, h_z, h_n = gh.chunk(3, dim=-1)
        r = torch.sigmoid(i_r + h_r)
        z = torch.sigmoid(i_z + h_z)
        n = torch.tanh(i_n + r * h_n)
        return (1.0 - z) * n + z * h

    h = cell(table[prefix_ids[:, 0]], h)
    out = torch.empty(B, steps, dtype=torch.long)
    for step in range(steps):
        rank_state = F.linear(h, w_rank)
        logits = base_logits[:, step, :] + alpha[step] * F.linear(rank_state, Vr)
        if prior is not None and beta[step] != 0.0:
            logits = logits - beta[step] * prior.view(1, -1)
        tok = torch.argmax(logits, dim=-1)
        out[:, step] = tok
        if step + 1 < steps:
            h = cell(table[tok], h)
    return out


def markov_rollout(prev_ids, base_logits, emb, lm_head, prior, alpha, beta) -> torch.Tensor:
    """MarkovDeLSGraphRunner._forward_impl's torch path (code/kernel/markov_dels.py:285-301),
    on the host: the previous token's embedding row as the rank state, base + alpha *
    low-rank - beta * prior, argmax, per step."""
    B, steps, _ = base_logits.shape
    cur = prev_ids[:, 0]
    out = torch.empty(B, steps, dtype=torch.long)
    for step in range(steps):
        rank_state = F.embedding(cur, emb)
        logits = base_logits[:, step, :] + alpha[step] * F.linear(rank_state, lm_head)
        if prior is not None and beta[step] != 0.0:
            logits = logits - beta[step] * prior.view(1, -1)
        cur = torch.argmax(logits, dim=-1)
        out[:, step] = cur
    return out


def domino_rollout(prefix_ids, hiddens, base_logits, table, w_hh, w_z, w_s, fc2, alpha) -> torch.Tensor:
    """DraftCorrectionGraphRunner._forward_impl's torch path (code/kernel/domino.py:399-451,
    bias-free released head: SiLU middle, GRU without biases), on the host."""
    B, steps, _ = base_logits.shape
    G = w_hh.shape[1]
    z_all = F.linear(hiddens, w_z)
    h = torch.zeros(B, G, dtype=base_logits.dtype)

    def cell(gi, h):
        gh = F.linear(h, w_hh)
        i_r, i_z, i_n = gi.chunk(3, dim=-1)
        h_r, h_z, h_n = gh.chunk(3, dim=-1)
        r = torch.sigmoid(i_r + h_r)
        z = torch.sigmoid(i_z + h_z)
        n = torch.tanh(i_n + r * h_n)
        return (1.0 - z) * n + z * h

    for p in range(prefix_ids.shape[1]):
        h = cell(table[prefix_ids[:, p]], h)
    out = torch.empty(B, steps, dtype=torch.long)
    for t in range(steps):
        mid = F.silu(z_all[:, t, :] + F.linear(h, w_s))
        logits = base_logits[:, t, :] + alpha * F.linear(mid, fc2)
        tok = torch.argmax(logits, dim=-1)
        out[:, t] = tok
        if t + 1 < steps:
            h = cell(table[tok], h)
    return out


@torch.inference_mode()
def rnn_rank_states(x, w_in, w_s, bias, T: int) -> torch.Tensor:
    """Rank states of the input-projected RNN head for rows x [n_seq * T, H] in [seq, t]
    order: s_t = tanh(W_in x_t + W_s s_(t-1) + b), s_0 = 0, in fp32, returned in x's dtype.
    The reference has no such head (only the GRU form); this restates the workload's own
    formula for the CPU baseline."""
    n_seq = x.shape[0] // T
    u = F.linear(x.float(), w_in.float()).view(n_seq, T, -1) + bias.float()
    s = torch.zeros(n_seq, w_s.shape[0], dtype=torch.float32)
    out = torch.empty_like(u)
    for t in range(T):
        s = torch.tanh(u[:, t] + F.linear(s, w_s.float()))
        out[:, t] = s
    return out.view(n_seq * T, -1).to(x.dtype)
