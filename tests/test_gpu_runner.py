"""The drop-in graph runners (kernel/dels.py, kernel/markov_dels.py) against the
reference's own runner outputs (tests/golden/runners.npz) and the oracle rollout.
Needs a B200.  After a step whose exact top-2 gap is below the tolerance the greedy
rollouts may legitimately diverge, so each row is compared up to that step."""

from __future__ import annotations

import json
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import dels_oracle as O

pytestmark = pytest.mark.gpu


def _head(dev, V, E, G, r, act, weights):
    import dels as D

    target = types.SimpleNamespace(model=types.SimpleNamespace(embed_tokens=nn.Embedding(V, E)),
                                   lm_head=nn.Linear(G, V, bias=False))
    head = D.DeLSLocalHead(target_model=target, vocab_size=V, embed_dim=E, gru_hidden_dim=G, low_rank_dim=r,
                           lm_head_mode="low_rank", rank_activation=act, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        head.embed_tokens.weight.copy_(torch.from_numpy(weights["embed"]).to(dev))
        head.prefix_gru.weight_ih_l0.copy_(torch.from_numpy(weights["w_ih"]).to(dev))
        head.prefix_gru.weight_hh_l0.copy_(torch.from_numpy(weights["w_hh"]).to(dev))
        head.rank_proj.weight.copy_(torch.from_numpy(weights["w_rank"]).to(dev))
        head.low_rank_lm_head.weight.copy_(torch.from_numpy(weights["Vr"]).to(dev))
    return head


def _compare(ours, gaps, ref, thresh):
    n = 0
    for b in range(ours.shape[0]):
        for t in range(ours.shape[1]):
            if gaps[b, t] <= thresh:
                break
            assert ours[b, t] == ref[b, t], (b, t, ours[b], ref[b])
            n += 1
    return n


@pytest.mark.parametrize("overlap", ["1", "split", "0"])
def test_dels_runner_matches_reference_fixture(cuda_device, golden_dir, monkeypatch, overlap):
    """The three small-batch schedules: the GRU gates fused into the rank projection or a
    gates kernel before the rank GEMV, both with the next step's W_hh h on the scorer's
    helper warps, and the GRU step kernel first."""
    from kernel.dels import DeLSGraphRunner

    monkeypatch.setenv("DELS_RUNNER_OVERLAP_ROWS", "64" if overlap == "1" else "0")
    monkeypatch.setenv("DELS_RUNNER_SPLIT_GRU", "0" if overlap == "0" else "1")
    g = np.load(golden_dir / "runners.npz")
    total = 0
    for c in json.loads(str(g["meta"])):
        n = c["name"]
        w = {k: g[f"{n}_{k}"] for k in ("embed", "w_ih", "w_hh", "w_rank", "Vr")}
        head = _head(cuda_device, c["V"], c["E"], c["G"], c["r"], c["activation"], w)
        prior = torch.from_numpy(g[f"{n}_prior_bf16"]).to(cuda_device) if c["prior"] else None
        runner = DeLSGraphRunner(local_head=head, batch_size=c["B"], steps=c["steps"], vocab_size=c["V"],
                                 alpha_values=list(g[f"{n}_alpha"]), beta_values=list(g[f"{n}_beta"]),
                                 baseline_logits=prior, device=cuda_device)
        base = torch.from_numpy(g[f"{n}_base"]).to(cuda_device).to(torch.bfloat16)
        prefix = torch.from_numpy(g[f"{n}_prefix"]).to(cuda_device)
        out = runner(prefix, base).cpu().numpy()
        assert out.shape == (c["B"], c["steps"])
        toks, gaps = O.dels_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_base"], embed=w["embed"], w_ih=w["w_ih"], w_hh=w["w_hh"], w_rank=w["w_rank"],
            Vr=w["Vr"], prior=None if prior is None else g[f"{n}_prior_bf16"], alpha=g[f"{n}_alpha"],
            beta=g[f"{n}_beta"], activation=c["activation"], bf16=True,
        )
        # the oracle's bf16-storage rollout (the reference's Triton-path semantics) ...
        total += _compare(out, gaps, toks, 1e-2)
        # ... and the reference runner's own bf16 output, away from its rounding noise
        _compare(out, gaps, g[f"{n}_tokens_bf16"], 0.05)
        # replay with other inputs: static buffers are refreshed on every call
        out2 = runner(torch.flip(prefix, [0]), torch.flip(base, [0])).cpu().numpy()
        toks2, gaps2 = O.dels_runner_rollout(
            np.flip(g[f"{n}_prefix"], 0), np.flip(g[f"{n}_base"], 0), embed=w["embed"], w_ih=w["w_ih"],
            w_hh=w["w_hh"], w_rank=w["w_rank"], Vr=w["Vr"], prior=None if prior is None else g[f"{n}_prior_bf16"],
            alpha=g[f"{n}_alpha"], beta=g[f"{n}_beta"], activation=c["activation"], bf16=True,
        )
        _compare(out2, gaps2, toks2, 1e-2)
    assert total >= 15


def test_markov_runner_matches_reference_fixture(cuda_device, golden_dir):
    import dels as D
    from kernel.markov_dels import MarkovDeLSGraphRunner

    g = np.load(golden_dir / "runners.npz")
    for c in json.loads(str(g["meta"])):
        n = c["name"]
        emb = torch.from_numpy(g[f"{n}_markov_embedding"])
        head = D.MarkovDeLSLocalHead(embedding_weight=emb, lm_head_weight=torch.from_numpy(g[f"{n}_Vr"]),
                                     dtype=torch.bfloat16, device=cuda_device)
        prior = torch.from_numpy(g[f"{n}_prior_bf16"]).to(cuda_device) if c["prior"] else None
        runner = MarkovDeLSGraphRunner(local_head=head, batch_size=c["B"], steps=c["steps"], vocab_size=c["V"],
                                       alpha_values=list(g[f"{n}_alpha"]), beta_values=list(g[f"{n}_beta"]),
                                       baseline_logits=prior, device=cuda_device)
        out = runner(torch.from_numpy(g[f"{n}_prefix"]).to(cuda_device),
                     torch.from_numpy(g[f"{n}_base"]).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
        toks, gaps = O.markov_runner_rollout(g[f"{n}_prefix"], g[f"{n}_base"], embedding=g[f"{n}_markov_embedding"],
                                             lm_head=g[f"{n}_Vr"], prior=None if prior is None else
                                             g[f"{n}_prior_bf16"], alpha=g[f"{n}_alpha"], beta=g[f"{n}_beta"])
        _compare(out, gaps, toks, 1e-2)
        _compare(out, gaps, g[f"{n}_markov_tokens_bf16"], 0.05)


def test_runner_validation_errors(cuda_device):
    from kernel.dels import DeLSGraphRunner

    with pytest.raises(ValueError, match="steps > 0"):
        DeLSGraphRunner(local_head=None, batch_size=1, steps=0, vocab_size=10, alpha_values=[], beta_values=[],
                        baseline_logits=None, device=cuda_device)
    with pytest.raises(ValueError, match="must match steps"):
        DeLSGraphRunner(local_head=None, batch_size=1, steps=2, vocab_size=10, alpha_values=[1.0], beta_values=[1, 1],
                        baseline_logits=None, device=cuda_device)
    with pytest.raises(ValueError, match="requires baseline_logits"):
        DeLSGraphRunner(local_head=None, batch_size=1, steps=1, vocab_size=10, alpha_values=[1.0], beta_values=[0.5],
                        baseline_logits=None, device=cuda_device)


def test_runner_full_vocab_b1(cuda_device):
    """Released head shapes (V=151936, E=256, G=1024, r=256), batch 1, 14 steps."""
    from kernel.dels import DeLSGraphRunner

    rng = np.random.default_rng(21)
    V, E, G, r, steps = 151936, 256, 1024, 256, 14
    w = {
        "embed": O.bf16_round((rng.standard_normal((V, E)) * 0.5).astype(np.float32)),
        "w_ih": O.bf16_round((rng.standard_normal((3 * G, E)) * 0.05).astype(np.float32)),
        "w_hh": O.bf16_round((rng.standard_normal((3 * G, G)) * 0.03).astype(np.float32)),
        "w_rank": O.bf16_round((rng.standard_normal((r, G)) * 0.05).astype(np.float32)),
        "Vr": O.bf16_round((rng.standard_normal((V, r)) * 0.05).astype(np.float32)),
    }
    head = _head(cuda_device, V, E, G, r, "identity", w)
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = list(np.linspace(0.9, 0.3, steps))
    beta = list(np.linspace(0.3, 0.1, steps))
    runner = DeLSGraphRunner(local_head=head, batch_size=1, steps=steps, vocab_size=V, alpha_values=alpha,
                             beta_values=beta, baseline_logits=torch.from_numpy(prior).to(cuda_device),
                             device=cuda_device)
    base = O.bf16_round(rng.standard_normal((1, steps, V)).astype(np.float32))
    prefix = np.array([[12345]])
    out = runner(torch.from_numpy(prefix).to(cuda_device), torch.from_numpy(base).to(cuda_device).to(torch.bfloat16))
    table = runner._gru_input_proj_table.float().cpu().numpy()  # bf16 F.linear(embed, W_ih) on the GPU
    toks, gaps = O.dels_runner_rollout(prefix, base, embed=None, w_ih=None, w_hh=w["w_hh"], w_rank=w["w_rank"],
                                       Vr=w["Vr"], prior=prior, alpha=alpha, beta=beta, bf16=True, table=table)
    assert _compare(out.cpu().numpy(), gaps, toks, 1e-2) >= 3


@pytest.mark.parametrize("B", [1, 3, 4, 5, 8])
def test_scorer_with_next_gru_projection(cuda_device, B):
    """dels_fused_argmax_base_gru_bf16: the same tokens as the plain base-logit scorer, and
    gh_out within one bf16 rounding of bf16(W_hh h + b_hh) (helper warps' fp32 sums)."""
    from dels_b200 import ops

    rng = np.random.default_rng(90 + B)
    V, r, G = 5003, 64, 256
    base = torch.from_numpy(O.bf16_round(rng.standard_normal((B, V)).astype(np.float32))).to(cuda_device)
    s = torch.from_numpy(O.bf16_round((rng.standard_normal((B, r)) * 0.3).astype(np.float32))).to(cuda_device)
    Vr = torch.from_numpy(O.bf16_round((rng.standard_normal((V, r)) * 0.3).astype(np.float32))).to(cuda_device)
    prior = torch.from_numpy(O.bf16_round(O.zipf_log_prior(V).astype(np.float32))).to(cuda_device)
    beta = torch.tensor([0.2], device=cuda_device)
    w_hh = O.bf16_round((rng.standard_normal((3 * G, G)) * 0.1).astype(np.float32))
    b_hh = O.bf16_round(rng.standard_normal(3 * G).astype(np.float32))
    h = O.bf16_round(rng.standard_normal((B, G)).astype(np.float32))
    bf = lambda a: torch.from_numpy(a).to(cuda_device).to(torch.bfloat16)  # noqa: E731
    base, s, Vr = base.to(torch.bfloat16), s.to(torch.bfloat16), Vr.to(torch.bfloat16)
    ws = ops.Workspace(1 << 12, cuda_device)
    ref = ops.fused_argmax_base_bf16(base, s, Vr, prior, beta, n_pos=1, ws=ws)
    out = ops.ScoreOut(tokens=torch.empty(B, dtype=torch.int64, device=cuda_device), scores=None,
                       keys=torch.empty(B, dtype=torch.int64, device=cuda_device))
    gh = torch.full((B, 3 * G), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    ops.fused_argmax_base_gru_bf16(base, s, Vr, prior, beta, bf(w_hh), bf(b_hh), bf(h), gh, out=out, ws=ws)
    ws.check()
    assert torch.equal(out.tokens, ref.tokens)
    exact = h.astype(np.float64) @ w_hh.astype(np.float64).T + b_hh.astype(np.float64)
    got = gh.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.mean(got == O.bf16_round(exact.astype(np.float32))) > 0.99
    np.testing.assert_allclose(got, exact, rtol=2 ** -7, atol=1e-3)


@pytest.mark.parametrize("B", [1, 3])
def test_gru_gates_from_packed_keys(cuda_device, B):
    """The fused GRU-gates entry points take the previous step's packed argmax keys in
    place of token ids (token_keys): h, s_scaled and the reset keys are bit-identical to
    the token-id call, and a keys-only scorer call plus one keys decode gives the tokens
    of the in-kernel decode."""
    from dels_b200 import ops

    rng = np.random.default_rng(70 + B)
    dev = cuda_device
    V, G, r, M = 4099, 256, 64, 96
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(torch.bfloat16)  # noqa: E731
    table = bf(rng.standard_normal((V, 3 * G)) * 0.5)
    gh = bf(rng.standard_normal((B, 3 * G)) * 0.5)
    h_in = bf(rng.standard_normal((B, G)))
    w_rank = bf(rng.standard_normal((r, G)) * 0.05)
    w_s = bf(rng.standard_normal((M, G)) * 0.05)
    z = bf(rng.standard_normal((B, M)))
    alpha = torch.tensor([0.7], device=dev)
    # keys of a keys-only scorer call over random base logits; the decoded tokens feed the
    # token-id path
    base = bf(rng.standard_normal((B, V)))
    s0 = bf(rng.standard_normal((B, r)) * 0.3)
    Vr = bf(rng.standard_normal((V, r)) * 0.3)
    prior = torch.from_numpy(O.bf16_round(O.zipf_log_prior(V).astype(np.float32))).to(dev)
    beta = torch.tensor([0.2], device=dev)
    ws = ops.Workspace(1 << 12, dev)
    ref = ops.fused_argmax_base_bf16(base, s0, Vr, prior, beta, n_pos=1, ws=ws)
    keys_only = ops.ScoreOut(tokens=None, scores=None, keys=torch.empty(B, dtype=torch.int64, device=dev))
    ops.fused_argmax_base_bf16(base, s0, Vr, prior, beta, n_pos=1, out=keys_only, ws=ws)
    tok, _ = ops.keys_decode(keys_only.keys, with_scores=False)
    assert torch.equal(tok, ref.tokens)
    assert torch.equal(keys_only.keys, ref.keys)
    for entry in ("rank", "correction"):
        outs = []
        for as_keys in (False, True):
            h_out = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
            width = r if entry == "rank" else M
            s_scaled = torch.empty(B, width, dtype=torch.bfloat16, device=dev)
            k_reset = torch.zeros(B, dtype=torch.int64, device=dev)
            src = keys_only.keys if as_keys else ref.tokens
            if entry == "rank":
                ops.gru_rank_gemv(src, table, gh, h_in, h_out, w_rank, alpha, s_scaled, keys=k_reset, ws=ws,
                                  tokens_are_keys=as_keys)
            else:
                ops.gru_correction_mid(src, table, gh, h_in, h_out, w_s, z, alpha, s_scaled, keys=k_reset, ws=ws,
                                       tokens_are_keys=as_keys)
            outs.append((h_out, s_scaled, k_reset))
        torch.cuda.synchronize()
        for a, b in zip(*outs):
            assert torch.equal(a, b), entry
    ws.check()


@pytest.mark.parametrize("B", [5, 8])
def test_runner_split_schedule_up_to_8_rows(cuda_device, monkeypatch, B):
    """The split schedule (gates kernel, rank GEMV, scorer whose helper warps compute the
    next W_hh h) at 5-8 rows, where the scorer stages its epilogue operands: tokens against
    the oracle rollout."""
    from kernel.dels import DeLSGraphRunner

    monkeypatch.setenv("DELS_RUNNER_SPLIT_ROWS", "8")
    rng = np.random.default_rng(120 + B)
    V, E, G, r, steps = 2003, 40, 64, 32, 4
    w = {
        "embed": O.bf16_round((rng.standard_normal((V, E)) * 0.5).astype(np.float32)),
        "w_ih": O.bf16_round((rng.standard_normal((3 * G, E)) * 0.2).astype(np.float32)),
        "w_hh": O.bf16_round((rng.standard_normal((3 * G, G)) * 0.2).astype(np.float32)),
        "w_rank": O.bf16_round((rng.standard_normal((r, G)) * 0.3).astype(np.float32)),
        "Vr": O.bf16_round((rng.standard_normal((V, r)) * 0.3).astype(np.float32)),
    }
    head = _head(cuda_device, V, E, G, r, "identity", w)
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = list(np.linspace(0.9, 0.5, steps))
    beta = list(np.linspace(0.3, 0.1, steps))
    runner = DeLSGraphRunner(local_head=head, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                             beta_values=beta, baseline_logits=torch.from_numpy(prior).to(cuda_device),
                             device=cuda_device)
    assert runner._split_gru and runner._keys_only
    base = O.bf16_round(rng.standard_normal((B, steps, V)).astype(np.float32))
    prefix = rng.integers(0, V, (B, 1))
    out = runner(torch.from_numpy(prefix).to(cuda_device),
                 torch.from_numpy(base).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    toks, gaps = O.dels_runner_rollout(prefix, base, embed=w["embed"], w_ih=w["w_ih"], w_hh=w["w_hh"],
                                       w_rank=w["w_rank"], Vr=w["Vr"], prior=prior, alpha=alpha, beta=beta,
                                       bf16=True)
    assert _compare(out, gaps, toks, 1e-2) >= B * steps // 2


@pytest.mark.parametrize("B", [4, 5, 12, 20, 48, 64])
def test_runner_batches(cuda_device, B):
    """Batch sizes past the fixtures': the plain (<= 4 rows) and staged skinny scorers (16- and
    32-column row tiles), the 128-row tile scorer (33..128 rows) and the GRU step's loop over
    16-row chunks, each against the oracle rollout."""
    from kernel.dels import DeLSGraphRunner

    rng = np.random.default_rng(100 + B)
    V, E, G, r, steps = 2003, 40, 64, 32, 4
    w = {
        "embed": O.bf16_round((rng.standard_normal((V, E)) * 0.5).astype(np.float32)),
        "w_ih": O.bf16_round((rng.standard_normal((3 * G, E)) * 0.2).astype(np.float32)),
        "w_hh": O.bf16_round((rng.standard_normal((3 * G, G)) * 0.2).astype(np.float32)),
        "w_rank": O.bf16_round((rng.standard_normal((r, G)) * 0.3).astype(np.float32)),
        "Vr": O.bf16_round((rng.standard_normal((V, r)) * 0.3).astype(np.float32)),
    }
    head = _head(cuda_device, V, E, G, r, "identity", w)
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = list(np.linspace(0.9, 0.5, steps))
    beta = list(np.linspace(0.3, 0.1, steps))
    runner = DeLSGraphRunner(local_head=head, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                             beta_values=beta, baseline_logits=torch.from_numpy(prior).to(cuda_device),
                             device=cuda_device)
    base = O.bf16_round(rng.standard_normal((B, steps, V)).astype(np.float32))
    prefix = rng.integers(0, V, (B, 1))
    out = runner(torch.from_numpy(prefix).to(cuda_device),
                 torch.from_numpy(base).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    toks, gaps = O.dels_runner_rollout(prefix, base, embed=w["embed"], w_ih=w["w_ih"], w_hh=w["w_hh"],
                                       w_rank=w["w_rank"], Vr=w["Vr"], prior=prior, alpha=alpha, beta=beta,
                                       bf16=True)
    assert _compare(out, gaps, toks, 1e-2) >= B * steps // 2


@pytest.mark.parametrize("schedule", ["fused", "materialised"])
def test_fused_long_logit_runner_matches_oracle(cuda_device, monkeypatch, schedule):
    """DeLSFusedGraphRunner from the hidden states: long logits computed inside each step's
    scorer (never rounded to bf16), or by one GEMM per call into the runner's own bf16
    buffer (the schedule for small batches)."""
    from kernel.dels import DeLSFusedGraphRunner

    monkeypatch.setenv("DELS_FUSED_RUNNER_ROWS", "1" if schedule == "fused" else "1000000")
    rng = np.random.default_rng(31)
    V, E, G, r, H, B, steps = 3001, 32, 64, 32, 256, 3, 6
    w = {
        "embed": O.bf16_round((rng.standard_normal((V, E)) * 0.5).astype(np.float32)),
        "w_ih": O.bf16_round((rng.standard_normal((3 * G, E)) * 0.2).astype(np.float32)),
        "w_hh": O.bf16_round((rng.standard_normal((3 * G, G)) * 0.2).astype(np.float32)),
        "w_rank": O.bf16_round((rng.standard_normal((r, G)) * 0.3).astype(np.float32)),
        "Vr": O.bf16_round((rng.standard_normal((V, r)) * 0.3).astype(np.float32)),
    }
    W = O.bf16_round((rng.standard_normal((V, H)) * 0.06).astype(np.float32))
    hid = O.bf16_round(rng.standard_normal((B, steps, H)).astype(np.float32))
    head = _head(cuda_device, V, E, G, r, "silu", w)
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = list(np.linspace(0.9, 0.4, steps))
    beta = list(np.linspace(0.1, 0.3, steps))
    runner = DeLSFusedGraphRunner(local_head=head, target_lm_head_weight=torch.from_numpy(W).to(cuda_device),
                                  batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha, beta_values=beta,
                                  baseline_logits=torch.from_numpy(prior).to(cuda_device), device=cuda_device)
    prefix = np.array([[5], [77], [2999]])
    out = runner(torch.from_numpy(prefix).to(cuda_device),
                 torch.from_numpy(hid).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    assert runner._fused == (schedule == "fused")
    base = np.einsum("bsh,vh->bsv", hid.astype(np.float64), W.astype(np.float64))  # exact
    if schedule == "materialised":
        base = O.bf16_round(base.astype(np.float32))  # the bf16 long logits, as the reference feeds them
    toks, gaps = O.dels_runner_rollout(prefix, base, embed=w["embed"], w_ih=w["w_ih"], w_hh=w["w_hh"],
                                       w_rank=w["w_rank"], Vr=w["Vr"], prior=prior, alpha=alpha, beta=beta,
                                       activation="silu", bf16=True)
    assert _compare(out, gaps, toks, 1e-2) >= 3


def test_runners_odd_widths(cuda_device):
    """Rank width 12 and embedding width 20 (not multiples of 8): the runners carry them
    zero-padded; results must still match the oracle."""
    from kernel.dels import DeLSGraphRunner
    from kernel.markov_dels import MarkovDeLSGraphRunner

    import dels as D

    rng = np.random.default_rng(77)
    V, E, G, r, B, steps = 900, 20, 24, 12, 2, 5
    w = {
        "embed": O.bf16_round((rng.standard_normal((V, E)) * 0.5).astype(np.float32)),
        "w_ih": O.bf16_round((rng.standard_normal((3 * G, E)) * 0.2).astype(np.float32)),
        "w_hh": O.bf16_round((rng.standard_normal((3 * G, G)) * 0.2).astype(np.float32)),
        "w_rank": O.bf16_round((rng.standard_normal((r, G)) * 0.3).astype(np.float32)),
        "Vr": O.bf16_round((rng.standard_normal((V, r)) * 0.3).astype(np.float32)),
    }
    base = O.bf16_round(rng.standard_normal((B, steps, V)).astype(np.float32))
    prefix = rng.integers(0, V, (B, 1))
    alpha = [0.9, 0.8, 0.7, 0.6, 0.5]
    beta = [0.0] * steps
    head = _head(cuda_device, V, E, G, r, "silu", w)
    runner = DeLSGraphRunner(local_head=head, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                             beta_values=beta, baseline_logits=None, device=cuda_device)
    out = runner(torch.from_numpy(prefix).to(cuda_device),
                 torch.from_numpy(base).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    toks, gaps = O.dels_runner_rollout(prefix, base, embed=w["embed"], w_ih=w["w_ih"], w_hh=w["w_hh"],
                                       w_rank=w["w_rank"], Vr=w["Vr"], prior=None, alpha=alpha, beta=beta,
                                       activation="silu", bf16=True)
    assert _compare(out, gaps, toks, 1e-2) >= 5
    emb_r = O.bf16_round((rng.standard_normal((V, r)) * 0.5).astype(np.float32))
    mhead = D.MarkovDeLSLocalHead(embedding_weight=torch.from_numpy(emb_r).to(torch.bfloat16),
                                  lm_head_weight=torch.from_numpy(w["Vr"]).to(torch.bfloat16), dtype=torch.bfloat16,
                                  device=cuda_device)
    mrunner = MarkovDeLSGraphRunner(local_head=mhead, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                                    beta_values=beta, baseline_logits=None, device=cuda_device)
    mout = mrunner(torch.from_numpy(prefix).to(cuda_device),
                   torch.from_numpy(base).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    mtoks, mgaps = O.markov_runner_rollout(prefix, base, embedding=emb_r, lm_head=w["Vr"], prior=None, alpha=alpha,
                                           beta=beta)
    assert _compare(mout, mgaps, mtoks, 1e-2) >= 5


@pytest.mark.parametrize("B", [1, 2, 3, 5, 8, 9, 16, 17, 40])
def test_small_batch_gemvs_every_rows_per_pass(cuda_device, B):
    """The GRU step and the rank GEMV at batches that select each of their compiled row
    counts (1, 2, 4, 8 and 16 rows per shared-memory pass) and the loop over 16-row passes
    (17, 40), against the oracle: gh = bf16(W_hh h), the gates in fp32, h' in bf16, then
    s = bf16(SiLU(bf16(W_rank h'))) and bf16(alpha_p s)."""
    from dels_b200 import ops

    rng = np.random.default_rng(700 + B)
    V, G, r, n_pos = 301, 256, 96, 5
    dev = cuda_device
    table = O.bf16_round((rng.standard_normal((V, 3 * G)) * 0.5).astype(np.float32))
    w_hh = O.bf16_round((rng.standard_normal((3 * G, G)) * 0.05).astype(np.float32))
    h_in = O.bf16_round((rng.standard_normal((B, G)) * 0.5).astype(np.float32))
    w_rank = O.bf16_round((rng.standard_normal((r, G)) * 0.1).astype(np.float32))
    tokens = rng.integers(0, V, B)
    alpha = np.linspace(0.9, 0.4, n_pos)
    bf = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731

    h_out = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
    ops.gru_step(torch.from_numpy(tokens).to(dev), bf(table), bf(w_hh), bf(h_in), h_out)
    gh = O.bf16_round((h_in.astype(np.float64) @ w_hh.astype(np.float64).T).astype(np.float32))
    ref_h = O.bf16_round(O.gru_cell(table[tokens], gh, h_in).astype(np.float32))
    got_h = h_out.float().cpu().numpy()
    assert np.mean(got_h == ref_h) > 0.98
    np.testing.assert_allclose(got_h, ref_h, rtol=2 ** -7, atol=2e-3)

    s_scaled = torch.empty(B, r, dtype=torch.bfloat16, device=dev)
    s_out = torch.empty(B, r, dtype=torch.bfloat16, device=dev)
    ops.rank_gemv(h_out, bf(w_rank), torch.from_numpy(alpha.astype(np.float32)).to(dev), s_scaled, n_pos=n_pos,
                  activation="silu", s_out=s_out)
    got_s = s_out.float().cpu().numpy()
    ref_s = O.rank_state_bf16(got_h, w_rank, "silu")
    assert np.mean(got_s == ref_s) > 0.98
    np.testing.assert_allclose(got_s, ref_s, rtol=2 ** -7, atol=2e-3)
    pos = np.arange(B) % n_pos
    ref_scaled = O.bf16_round((alpha[pos][:, None].astype(np.float32) * got_s).astype(np.float32))
    np.testing.assert_array_equal(s_scaled.float().cpu().numpy(), ref_scaled)


@pytest.mark.parametrize("B", [12, 33, 64])
def test_gru_step_tc_matches_linear_then_gates(cuda_device, B):
    """The tensor-core GRU step whose split-K finalisation evaluates the gates gives h_out
    bit-identical to dels_linear_bf16 followed by dels_gru_gates_bf16 (with and without
    b_hh), and matches the oracle cell."""
    from dels_b200 import ops

    dev = cuda_device
    rng = np.random.default_rng(1200 + B)
    V, G = 503, 256
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)  # noqa: E731
    table = bf(rng.standard_normal((V, 3 * G)) * 0.5)
    w_hh = bf(rng.standard_normal((3 * G, G)) * 0.05)
    b_hh = bf(rng.standard_normal(3 * G) * 0.1)
    h_in = bf(rng.standard_normal((B, G)) * 0.5)
    tokens = torch.from_numpy(rng.integers(0, V, B)).to(dev)
    for bias in (None, b_hh):
        ref = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
        gh = ops.linear_bf16(h_in, w_hh, bias)
        ops.gru_gates(tokens, table, gh, h_in, ref)
        out = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
        ops.gru_step_tc(tokens, table, w_hh, h_in, out, b_hh=bias)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    gh_ref = O.bf16_round((f(h_in).astype(np.float64) @ f(w_hh).astype(np.float64).T + f(b_hh)).astype(np.float32))
    cell = O.bf16_round(O.gru_cell(f(table)[tokens.cpu().numpy()], gh_ref, f(h_in)).astype(np.float32))
    np.testing.assert_allclose(f(out), cell, rtol=2 ** -7, atol=2e-3)


def test_gru_entry_points_read_packed_keys(cuda_device):
    """The GRU step, the tensor-core GRU step and the gates kernel give the same h whether
    the previous tokens come as ids or as the scorer's packed (score, index) keys."""
    from dels_b200 import ops

    dev = cuda_device
    rng = np.random.default_rng(1300)
    B, V, G = 10, 503, 128
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)  # noqa: E731
    table = bf(rng.standard_normal((V, 3 * G)) * 0.5)
    w_hh = bf(rng.standard_normal((3 * G, G)) * 0.05)
    h_in = bf(rng.standard_normal((B, G)) * 0.5)
    gh = bf(rng.standard_normal((B, 3 * G)) * 0.5)
    tok = rng.integers(0, V, B)
    ids = torch.from_numpy(tok).to(dev)
    keys = torch.from_numpy(O.pack_keys(rng.standard_normal(B).astype(np.float32), tok)).to(dev)
    for run in (lambda t, o, k: ops.gru_step(t, table, w_hh, h_in, o, tokens_are_keys=k),
                lambda t, o, k: ops.gru_step_tc(t, table, w_hh, h_in, o, tokens_are_keys=k),
                lambda t, o, k: ops.gru_gates(t, table, gh, h_in, o, tokens_are_keys=k)):
        a = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
        b = torch.empty(B, G, dtype=torch.bfloat16, device=dev)
        run(ids, a, False)
        run(keys, b, True)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
