"""The CPU baseline that bench.py times (oracle/reference_torch.py, a torch restatement of
the reference's host path) checked against the golden fixtures made from the reference
itself, so that the baseline computes the reference's answers.  CPU only; the oracle
supplies the top-2 gaps that decide which positions must agree exactly."""

from __future__ import annotations

import json

import numpy as np
import torch
import torch.nn.functional as F

from oracle import dels_oracle as O
from oracle import reference_torch as R


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_score_rows_fp32_matches_reference(golden_dir):
    g = np.load(golden_dir / "scorer.npz")
    checked = 0
    for c in json.loads(str(g["meta"])):
        if c["activation"] != "identity":
            continue  # the restatement carries the identity rank state only
        n, P = c["name"], c["P"]
        prior = g[f"{n}_prior_f32"] if c["prior"] else None
        pos = np.arange(c["B"] * P) % P
        tok = R.score_rows(_t(g[f"{n}_h"]), _t(g[f"{n}_W"]), _t(g[f"{n}_Ut"]), _t(g[f"{n}_Vr"]),
                           None if prior is None else _t(prior), g[f"{n}_alpha"][pos], g[f"{n}_beta"][pos]).numpy()
        _, _, gap = O.draft_score_f32(g[f"{n}_h"], g[f"{n}_W"], g[f"{n}_Ut"], g[f"{n}_Vr"], prior, g[f"{n}_alpha"],
                                      g[f"{n}_beta"], n_pos=P)
        ok = gap > 1e-5
        np.testing.assert_array_equal(tok[ok], g[f"{n}_tokens_f32"][ok])
        checked += int(ok.sum())
    assert checked >= 12


def _rollouts_agree(ours, gaps, ref, thresh):
    n = 0
    for b in range(ours.shape[0]):
        for t in range(ours.shape[1]):
            if gaps[b, t] <= thresh:
                break
            assert ours[b, t] == ref[b, t], (b, t)
            n += 1
    return n


def test_runner_rollout_fp32_matches_reference(golden_dir):
    g = np.load(golden_dir / "runners.npz")
    checked = 0
    for c in json.loads(str(g["meta"])):
        if c["activation"] != "identity":
            continue
        n = c["name"]
        prior = g[f"{n}_prior_f32"] if c["prior"] else None
        table = F.linear(_t(g[f"{n}_embed"]), _t(g[f"{n}_w_ih"]))
        ours = R.runner_rollout(_t(g[f"{n}_prefix"]), _t(g[f"{n}_base"]), table, _t(g[f"{n}_w_hh"]),
                                _t(g[f"{n}_w_rank"]), _t(g[f"{n}_Vr"]), None if prior is None else _t(prior),
                                list(g[f"{n}_alpha"]), list(g[f"{n}_beta"])).numpy()
        _, gaps = O.dels_runner_rollout(g[f"{n}_prefix"], g[f"{n}_base"], embed=g[f"{n}_embed"],
                                        w_ih=g[f"{n}_w_ih"], w_hh=g[f"{n}_w_hh"], w_rank=g[f"{n}_w_rank"],
                                        Vr=g[f"{n}_Vr"], prior=prior, alpha=g[f"{n}_alpha"], beta=g[f"{n}_beta"],
                                        activation="identity", bf16=False)
        checked += _rollouts_agree(ours, gaps, g[f"{n}_tokens_f32"], 1e-5)
    assert checked >= 10


def test_domino_rollout_fp32_matches_reference(golden_dir):
    g = np.load(golden_dir / "domino.npz")
    checked = 0
    for c in json.loads(str(g["meta"])):
        if c["bias"]:
            continue  # the restatement carries the released bias-free head
        n, H = c["name"], c["H"]
        w1 = g[f"{n}_embed_proj_0_weight"]
        table = F.linear(_t(g[f"{n}_embed"]), _t(g[f"{n}_prefix_gru_weight_ih_l0"]))
        ours = R.domino_rollout(_t(g[f"{n}_prefix"]), _t(g[f"{n}_hiddens"]), _t(g[f"{n}_base"]), table,
                                _t(g[f"{n}_prefix_gru_weight_hh_l0"]), _t(w1[:, :H]), _t(w1[:, H:]),
                                _t(g[f"{n}_embed_proj_2_weight"]), c["alpha"]).numpy()
        _, gaps = O.domino_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_hiddens"], g[f"{n}_base"], alpha=c["alpha"], bf16=False,
            embed=g[f"{n}_embed"], w_ih=g[f"{n}_prefix_gru_weight_ih_l0"], w_hh=g[f"{n}_prefix_gru_weight_hh_l0"],
            b_ih=None, b_hh=None, w1=w1, b1=None, fc2=g[f"{n}_embed_proj_2_weight"], b2=None)
        checked += _rollouts_agree(ours, gaps, g[f"{n}_tokens_f32"], 1e-5)
    assert checked >= 4


def test_rnn_rank_states_follow_the_recurrence():
    rng = np.random.default_rng(7)
    n_seq, T, H, r = 3, 5, 24, 8
    x = rng.standard_normal((n_seq * T, H)).astype(np.float32)
    w_in = (rng.standard_normal((r, H)) * 0.2).astype(np.float32)
    w_s = (rng.standard_normal((r, r)) * 0.3).astype(np.float32)
    b = rng.standard_normal(r).astype(np.float32)
    got = R.rnn_rank_states(_t(x), _t(w_in), _t(w_s), _t(b), T).numpy()
    want = np.empty((n_seq * T, r))
    for q in range(n_seq):
        s = np.zeros(r)
        for t in range(T):
            s = np.tanh(w_in.astype(np.float64) @ x[q * T + t] + w_s.astype(np.float64) @ s + b)
            want[q * T + t] = s
    np.testing.assert_allclose(got, want, atol=1e-5)
