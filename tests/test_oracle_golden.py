"""Pin the CPU oracle against fixtures produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import dels_oracle as O


def _load(golden_dir, name):
    return np.load(golden_dir / name, allow_pickle=False)


def test_schedules_match_reference(golden_dir):
    cases = json.loads((golden_dir / "schedules.json").read_text())
    assert len(cases) >= 8
    for c in cases:
        values = tuple(c["values"]) if c["is_tuple"] else c["values"]
        if "error" in c:
            with pytest.raises(ValueError) as ei:
                O.parse_scalar_schedule(values, c["steps"], name="DeLS alpha")
            assert str(ei.value) == c["error"]
        else:
            assert O.parse_scalar_schedule(values, c["steps"], name="DeLS alpha") == c["ok"]


def test_priors_match_reference(golden_dir):
    g = _load(golden_dir, "priors.npz")
    counts = g["counts"]
    V = int(g["vocab_size"])
    n = 0
    for key in g.files:
        if not key.endswith(("_f64", "_bf16")):
            continue
        sm = float(key.split("_s")[-1].split("_")[0])
        ours = O.log_unigram_prior(counts, V, sm)
        if key.endswith("_f64"):
            np.testing.assert_allclose(ours, g[key], rtol=0, atol=1e-12)
        else:
            np.testing.assert_array_equal(O.bf16_round(ours.astype(np.float32)), g[key].astype(np.float32))
        n += 1
    assert n == 24


def test_prior_errors():
    with pytest.raises(ValueError):
        O.log_unigram_prior(np.ones(10), 5)
    with pytest.raises(ValueError):
        O.log_unigram_prior(np.zeros(5), 5, smoothing=0.0)
    with pytest.raises(ValueError):
        O.log_unigram_prior(np.ones(5), 5, smoothing=-1.0)


def _scorer_cases(g):
    return json.loads(str(g["meta"]))


def test_scorer_fp32_matches_reference(golden_dir):
    g = _load(golden_dir, "scorer.npz")
    for c in _scorer_cases(g):
        n = c["name"]
        prior = g[f"{n}_prior_f32"] if c["prior"] else None
        tok, sc, gap = O.draft_score_f32(
            g[f"{n}_h"], g[f"{n}_W"], g[f"{n}_Ut"], g[f"{n}_Vr"], prior, g[f"{n}_alpha"], g[f"{n}_beta"],
            n_pos=c["P"],
        ) if c["activation"] == "identity" else (None, None, None)
        if tok is None:
            # fp32 SiLU rank state: apply the activation in fp32 like F.silu on fp32 tensors
            s = g[f"{n}_h"].astype(np.float64) @ g[f"{n}_Ut"].astype(np.float64).T
            s = s / (1.0 + np.exp(-s))
            pos = np.arange(c["B"] * c["P"]) % c["P"]
            sc = O.draft_scores(g[f"{n}_h"], g[f"{n}_W"], s, g[f"{n}_Vr"], prior, g[f"{n}_alpha"][pos],
                                g[f"{n}_beta"][pos])
            tok, gap = O.argmax_first(sc), O.top2_gap(sc)
        np.testing.assert_allclose(sc, g[f"{n}_final_f32"], rtol=0, atol=1e-5)
        ok = gap > 1e-5
        assert ok.mean() > 0.9
        np.testing.assert_array_equal(tok[ok], g[f"{n}_tokens_f32"][ok])


def test_scorer_bf16_matches_reference(golden_dir):
    """The reference's bf16 eager path rounds every intermediate tensor to bf16; the
    oracle keeps the mix exact.  Scores agree to bf16 rounding and tokens agree on
    every row whose exact top-2 gap exceeds that rounding."""
    g = _load(golden_dir, "scorer.npz")
    for c in _scorer_cases(g):
        n = c["name"]
        prior = g[f"{n}_prior_bf16"] if c["prior"] else None
        tok, sc, gap = O.draft_score_bf16(
            g[f"{n}_h"], g[f"{n}_W"], g[f"{n}_Ut"], g[f"{n}_Vr"], prior, g[f"{n}_alpha"], g[f"{n}_beta"],
            n_pos=c["P"], activation=c["activation"],
        )
        ref = g[f"{n}_final_bf16"].astype(np.float64)
        tol = 2.0 ** -6 * np.maximum(np.abs(sc), 1.0)
        assert np.all(np.abs(sc - ref) <= tol)
        ok = gap > 0.05
        assert ok.mean() > 0.5
        np.testing.assert_array_equal(tok[ok], g[f"{n}_tokens_bf16"][ok])


def _compare_rollout(ours, gaps, ref, thresh):
    """Positions agree until the first step whose oracle top-2 gap is below `thresh`
    (after a legitimate near-tie the greedy rollouts may part ways)."""
    compared = 0
    for b in range(ours.shape[0]):
        for t in range(ours.shape[1]):
            if gaps[b, t] <= thresh:
                break
            assert ours[b, t] == ref[b, t], (b, t)
            compared += 1
    return compared


def _runner_cases(g):
    return json.loads(str(g["meta"]))


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_dels_runner_matches_reference(golden_dir, mode):
    g = _load(golden_dir, "runners.npz")
    total = 0
    for c in _runner_cases(g):
        n = c["name"]
        prior = g[f"{n}_prior_{mode}"] if c["prior"] else None
        toks, gaps = O.dels_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_base"], embed=g[f"{n}_embed"], w_ih=g[f"{n}_w_ih"], w_hh=g[f"{n}_w_hh"],
            w_rank=g[f"{n}_w_rank"], Vr=g[f"{n}_Vr"], prior=prior, alpha=g[f"{n}_alpha"], beta=g[f"{n}_beta"],
            activation=c["activation"], bf16=(mode == "bf16"),
        )
        total += _compare_rollout(toks, gaps, g[f"{n}_tokens_{mode}"], 1e-5 if mode == "f32" else 0.05)
    assert total >= 20


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_markov_runner_matches_reference(golden_dir, mode):
    g = _load(golden_dir, "runners.npz")
    total = 0
    for c in _runner_cases(g):
        n = c["name"]
        prior = g[f"{n}_prior_{mode}"] if c["prior"] else None
        toks, gaps = O.markov_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_base"], embedding=g[f"{n}_markov_embedding"], lm_head=g[f"{n}_Vr"],
            prior=prior, alpha=g[f"{n}_alpha"], beta=g[f"{n}_beta"],
        )
        total += _compare_rollout(toks, gaps, g[f"{n}_markov_tokens_{mode}"], 1e-5 if mode == "f32" else 0.05)
    assert total >= 20


def domino_params(g, n, bias):
    """Oracle keyword arguments for Domino case n of tests/golden/domino.npz."""
    opt = (lambda k: g[f"{n}_{k}"]) if bias else (lambda k: None)
    return dict(
        embed=g[f"{n}_embed"], w_ih=g[f"{n}_prefix_gru_weight_ih_l0"], w_hh=g[f"{n}_prefix_gru_weight_hh_l0"],
        b_ih=opt("prefix_gru_bias_ih_l0"), b_hh=opt("prefix_gru_bias_hh_l0"), w1=g[f"{n}_embed_proj_0_weight"],
        b1=opt("embed_proj_0_bias"), fc2=g[f"{n}_embed_proj_2_weight"], b2=opt("embed_proj_2_bias"),
    )


@pytest.mark.parametrize("mode", ["f32", "bf16", "bf16_fused"])
def test_domino_runner_matches_reference(golden_dir, mode):
    """DraftCorrectionGraphRunner (code/kernel/domino.py:232-520): the torch path in fp32 /
    bf16 and the fused Triton step (run by Triton's CPU interpreter) against the oracle."""
    g = _load(golden_dir, "domino.npz")
    total = 0
    for c in _runner_cases(g):
        n = c["name"]
        toks, gaps = O.domino_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_hiddens"], g[f"{n}_base"], alpha=c["alpha"], bf16=(mode != "f32"),
            **domino_params(g, n, c["bias"]),
        )
        total += _compare_rollout(toks, gaps, g[f"{n}_tokens_{mode}"], 1e-5 if mode == "f32" else 0.05)
    assert total >= 12


def test_accept_matches_reference(golden_dir):
    g = _load(golden_dir, "accept.npz")
    draft = g["verify"][:, 1:]
    target = g["posterior"]
    acc, off = O.accept_offsets(draft, target)
    np.testing.assert_array_equal(acc, g["accept"])
    assert off[0] == 0 and off[-1] == g["accept"].sum()
    np.testing.assert_array_equal(np.diff(off), g["accept"])
    acc1, off1 = O.accept_offsets(draft, target, commit_extra=1)
    np.testing.assert_array_equal(np.diff(off1), g["accept"] + 1)
