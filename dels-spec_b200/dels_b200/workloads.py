"""Seeded synthetic inputs for the draft-scoring workloads.

The five workloads are the shapes the path is benchmarked on (a Qwen3-4B-shaped fp32
case, a Qwen3-8B-shaped bf16 case, a ragged continuous batch, an input-projected RNN
local head and a vocab-sharded large batch).  All tensors are generated on the target
device with ``torch.Generator(device).manual_seed(seed)`` in a fixed order, so every
process (and every rank) that asks for the same workload gets identical values.

Distributions: draft hidden states ~ N(0, 1); LM-head, local-head and RNN weights
~ N(0, 0.02); the log-unigram prior is Zipf(1.1) over token ids (token v has weight
(v+1)^-1.1), normalised and logged in float64, then rounded to bf16 for the bf16
workloads exactly as the reference's benchmark loads it
(``load_unigram_log_prior(..., dtype=torch.bfloat16)``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

VOCAB = 151936


@dataclass
class Workload:
    name: str
    dtype: torch.dtype
    rows: int
    H: int
    r: int
    V: int
    n_pos: int
    alpha: list[float]
    beta: list[float]
    seed: int
    tensors: dict[str, torch.Tensor] = field(default_factory=dict)

    def t(self, name: str) -> torch.Tensor:
        return self.tensors[name]


def zipf_log_prior(V: int, s: float = 1.1, device="cpu") -> torch.Tensor:
    k = torch.arange(1, V + 1, dtype=torch.float64, device=device)
    w = k.pow(-s)
    return torch.log(w / w.sum())


def linspace(a: float, b: float, n: int) -> list[float]:
    return [a + (b - a) * i / (n - 1) for i in range(n)] if n > 1 else [a]


def _randn(g: torch.Generator, shape, std: float, dtype, device) -> torch.Tensor:
    x = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    return x.to(dtype)


def dense_workload(
    name: str,
    *,
    rows: int,
    H: int,
    r: int,
    V: int = VOCAB,
    dtype=torch.bfloat16,
    alpha: list[float],
    beta: list[float],
    seed: int,
    device="cuda",
    v_slice: tuple[int, int] | None = None,
) -> Workload:
    """h [rows, H], W [V, H], w_rank [r, H] (= U^T), Vr [V, r], prior [V] fp32.

    With ``v_slice=(v0, v1)`` only that vocabulary slice of W / Vr / prior is kept
    (the full tensors are generated and sliced, so every shard sees the same values)."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h = _randn(g, (rows, H), 1.0, dtype, device)
    W = _randn(g, (V, H), 0.02, dtype, device)
    w_rank = _randn(g, (r, H), 0.02, dtype, device)
    Vr = _randn(g, (V, r), 0.02, dtype, device)
    prior = zipf_log_prior(V, device=device)
    prior = prior.to(dtype).to(torch.float32) if dtype == torch.bfloat16 else prior.to(torch.float32)
    if v_slice is not None:
        v0, v1 = v_slice
        W = W[v0:v1].contiguous()
        Vr = Vr[v0:v1].contiguous()
        prior = prior[v0:v1].contiguous()
    wl = Workload(name, dtype, rows, H, r, V, len(alpha), alpha, beta, seed)
    wl.tensors.update(
        h=h,
        W=W,
        w_rank=w_rank,
        Vr=Vr,
        prior=prior,
        alpha=torch.tensor(alpha, dtype=torch.float32, device=device),
        beta=torch.tensor(beta, dtype=torch.float32, device=device),
    )
    return wl


def cfg1(device="cuda", V: int = VOCAB) -> Workload:
    """Qwen3-4B shape, fp32: 16 rows, H=2560, r=64, alpha = beta = 0.3, seed 0."""
    return dense_workload("cfg1_qwen3_4b_fp32", rows=16, H=2560, r=64, V=V, dtype=torch.float32, alpha=[0.3],
                          beta=[0.3], seed=0, device=device)


def cfg2(device="cuda", V: int = VOCAB) -> Workload:
    """Qwen3-8B shape, bf16: 32 x 16 = 512 rows, H=4096, r=256, per-position schedules
    alpha_p = 0.5 -> 0.1, beta_p = 0.3 -> 0.0 over p = 0..15, seed 1."""
    return dense_workload("cfg2_qwen3_8b_bf16_b32x16", rows=512, H=4096, r=256, V=V, dtype=torch.bfloat16,
                          alpha=linspace(0.5, 0.1, 16), beta=linspace(0.3, 0.0, 16), seed=1, device=device)


def cfg5(device="cuda", V: int = VOCAB, v_slice=None, rows: int = 16384) -> Workload:
    """Vocab-sharded large batch: 1024 x 16 = 16384 rows, H=4096, r=256, alpha=beta=0.3, seed 4."""
    return dense_workload("cfg5_vocab_sharded_16384", rows=rows, H=4096, r=256, V=V, dtype=torch.bfloat16,
                          alpha=[0.3], beta=[0.3], seed=4, device=device, v_slice=v_slice)


def cfg3(device="cuda", V: int = VOCAB, n_seq: int = 256, P: int = 16, H: int = 4096, r: int = 256) -> Workload:
    """Ragged continuous batch, seed 2: draft [n_seq, P] and target [n_seq, P+1] uniform
    over the vocabulary, the first k ~ U{0..P} draft tokens forced equal to the target's;
    draft hidden [n_seq, P, H]; Qwen3-8B-shape scorer weights with cfg2's schedules."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(2)
    draft = torch.randint(0, V, (n_seq, P), generator=g, device=device)
    target = torch.randint(0, V, (n_seq, P + 1), generator=g, device=device)
    k = torch.randint(0, P + 1, (n_seq,), generator=g, device=device)
    j = torch.arange(P, device=device)[None, :]
    draft = torch.where(j < k[:, None], target[:, :P], draft)
    hidden = _randn(g, (n_seq, P, H), 1.0, torch.bfloat16, device)
    W = _randn(g, (V, H), 0.02, torch.bfloat16, device)
    w_rank = _randn(g, (r, H), 0.02, torch.bfloat16, device)
    Vr = _randn(g, (V, r), 0.02, torch.bfloat16, device)
    prior = zipf_log_prior(V, device=device).to(torch.bfloat16).to(torch.float32)
    alpha, beta = linspace(0.5, 0.1, P), linspace(0.3, 0.0, P)
    wl = Workload("cfg3_ragged_256seq", torch.bfloat16, n_seq * P, H, r, V, P, alpha, beta, 2)
    wl.tensors.update(
        draft=draft, target=target, k=k, hidden=hidden, W=W, w_rank=w_rank, Vr=Vr, prior=prior,
        alpha=torch.tensor(alpha, dtype=torch.float32, device=device),
        beta=torch.tensor(beta, dtype=torch.float32, device=device),
    )
    return wl


def cfg4(device="cuda", V: int = VOCAB, n_seq: int = 512, T: int = 16, H: int = 4096, r: int = 256) -> Workload:
    """Input-projected RNN local head, seed 3: x [n_seq*T, H] ~ N(0,1) (rows in [seq, t]
    order), W_in [r, H], W_s [r, r] ~ N(0, 0.02), bias b = 0 (unspecified by the
    workload, so zero), s_0 = 0; Vr [V, r], W [V, H]; alpha = beta = 0.3."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(3)
    x = _randn(g, (n_seq * T, H), 1.0, torch.bfloat16, device)
    w_in = _randn(g, (r, H), 0.02, torch.bfloat16, device)
    w_s = _randn(g, (r, r), 0.02, torch.bfloat16, device)
    W = _randn(g, (V, H), 0.02, torch.bfloat16, device)
    Vr = _randn(g, (V, r), 0.02, torch.bfloat16, device)
    prior = zipf_log_prior(V, device=device).to(torch.bfloat16).to(torch.float32)
    alpha, beta = [0.3] * T, [0.3] * T
    wl = Workload("cfg4_rnn_head_512x16", torch.bfloat16, n_seq * T, H, r, V, T, alpha, beta, 3)
    wl.tensors.update(
        x=x, w_in=w_in, w_s=w_s, bias=torch.zeros(r, dtype=torch.float32, device=device), W=W, Vr=Vr, prior=prior,
        alpha=torch.tensor(alpha, dtype=torch.float32, device=device),
        beta=torch.tensor(beta, dtype=torch.float32, device=device),
    )
    wl.n_seq, wl.T = n_seq, T  # type: ignore[attr-defined]
    return wl


def shard_range(V: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """Contiguous vocabulary slice of `rank`, boundaries rounded to `align` tokens."""
    per = math.ceil(V / world / align) * align
    v0 = min(V, rank * per)
    v1 = min(V, v0 + per)
    return v0, v1
