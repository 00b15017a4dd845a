"""The drop-in ``dels.py`` (dels-spec_b200/dels.py) against the reference's own loaders:
schedule parsing, the unigram prior, checkpoint-kind detection and the three local-head
modules on SpecForge-style checkpoints (tests/golden/ckpt, written and loaded by the
reference in tests/golden/make_golden.py).  CPU only."""

from __future__ import annotations

import json
import tempfile
import types
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn

import dels as D

CKPT = Path(__file__).resolve().parent / "golden" / "ckpt"


@pytest.fixture(scope="module")
def expected():
    return json.loads((CKPT / "expected.json").read_text())


@pytest.fixture(scope="module")
def outputs():
    return np.load(CKPT / "outputs.npz")


@pytest.fixture(scope="module")
def target():
    t = torch.load(CKPT / "target.pt")
    V, E = t["embed"].shape
    Hd = t["lm_head"].shape[1]
    model = types.SimpleNamespace(embed_tokens=nn.Embedding(V, E))
    tgt = types.SimpleNamespace(model=model, lm_head=nn.Linear(Hd, V, bias=False))
    with torch.no_grad():
        tgt.model.embed_tokens.weight.copy_(t["embed"])
        tgt.lm_head.weight.copy_(t["lm_head"])
    return tgt


def test_schedules_match_reference(golden_dir):
    for c in json.loads((golden_dir / "schedules.json").read_text()):
        values = tuple(c["values"]) if c["is_tuple"] else c["values"]
        if "error" in c:
            with pytest.raises(ValueError) as ei:
                D.parse_scalar_schedule(values, c["steps"], name="DeLS alpha")
            assert str(ei.value) == c["error"]
        else:
            assert D.parse_scalar_schedule(values, c["steps"], name="DeLS alpha") == c["ok"]


def test_prior_loader_matches_reference(golden_dir, tmp_path):
    g = np.load(golden_dir / "priors.npz")
    counts, V = g["counts"], int(g["vocab_size"])
    torch.save({"counts": torch.from_numpy(counts)}, tmp_path / "dict.pt")
    torch.save(torch.from_numpy(counts), tmp_path / "tensor.pt")
    np.savez(tmp_path / "c.npz", counts=counts)
    (tmp_path / "dir").mkdir()
    np.savez(tmp_path / "dir" / "loss_mask_unigram.npz", counts=counts)
    for tag, path in (("dict_pt", "dict.pt"), ("tensor_pt", "tensor.pt"), ("npz", "c.npz"), ("dir", "dir")):
        for sm in (1.0, 0.5, 0.0):
            for dtype, dname in ((torch.float64, "f64"), (torch.bfloat16, "bf16")):
                lp = D.load_unigram_log_prior(str(tmp_path / path), vocab_size=V, dtype=dtype,
                                              device=torch.device("cpu"), smoothing=sm)
                assert lp.shape == (1, 1, V) and lp.dtype == dtype
                np.testing.assert_array_equal(lp.to(torch.float64).reshape(-1).numpy(), g[f"{tag}_s{sm}_{dname}"])


def test_prior_loader_errors(tmp_path):
    with pytest.raises(ValueError, match="non-negative"):
        D.load_unigram_log_prior(str(tmp_path), vocab_size=3, dtype=torch.float32, device="cpu", smoothing=-1)
    with pytest.raises(ValueError, match="must contain"):
        D.load_unigram_log_prior(str(tmp_path), vocab_size=3, dtype=torch.float32, device="cpu")
    torch.save(torch.ones(5), tmp_path / "x.pt")
    with pytest.raises(ValueError, match="exceeds"):
        D.load_unigram_log_prior(str(tmp_path / "x.pt"), vocab_size=3, dtype=torch.float32, device="cpu")
    torch.save(torch.zeros(3), tmp_path / "z.pt")
    with pytest.raises(ValueError, match="no positive counts"):
        D.load_unigram_log_prior(str(tmp_path / "z.pt"), vocab_size=3, dtype=torch.float32, device="cpu",
                                 smoothing=0.0)
    (tmp_path / "bad.txt").write_text("1")
    with pytest.raises(ValueError, match="Unsupported unigram baseline path"):
        D.load_unigram_log_prior(str(tmp_path / "bad.txt"), vocab_size=3, dtype=torch.float32, device="cpu")


@pytest.mark.parametrize("name", ["direct_vocab", "target_factorized", "merged_head", "merged_head_target",
                                  "input_projection", "unexpected_tensor", "markov_merged", "markov_factorized",
                                  "position_mix", "unknown"])
def test_checkpoint_kind_matches_reference(name, expected):
    rec = expected[name]
    path = str(CKPT / f"{name}.pt")
    if "kind" in rec:
        assert D.detect_local_head_checkpoint_kind(path) == rec["kind"]
    else:
        with pytest.raises(ValueError) as ei:
            D.detect_local_head_checkpoint_kind(path)
        assert str(ei.value) == rec["kind_error"]


@pytest.mark.parametrize("name", ["direct_vocab", "target_factorized", "merged_head", "merged_head_target",
                                  "input_projection", "unexpected_tensor"])
def test_dels_local_head_matches_reference(name, expected, outputs, target):
    rec = expected[name]
    kw = {"merged_lm_head_path": str(CKPT / "merged_head_weight.pt")} if name.startswith("merged_head") else {}
    if "load_error" in rec:
        with pytest.raises(ValueError) as ei:
            D.DeLSLocalHead.from_checkpoint(checkpoint_path=str(CKPT / f"{name}.pt"), target_model=target,
                                            dtype=torch.float32, device=torch.device("cpu"), **kw)
        assert str(ei.value) == rec["load_error"]
        return
    m = D.DeLSLocalHead.from_checkpoint(checkpoint_path=str(CKPT / f"{name}.pt"), target_model=target,
                                        dtype=torch.float32, device=torch.device("cpu"), **kw)
    assert m.lm_head_mode == rec["lm_head_mode"]
    assert m.pure_draft_prefix_len == rec["pure"]
    assert m.shift_label == rec["shift_label"]
    assert m.rank_activation == rec["rank_activation"]
    hidden = torch.from_numpy(outputs["hidden"])
    tokens = torch.from_numpy(outputs["tokens"])
    torch.testing.assert_close(m.low_rank_lm_head.weight.detach(), torch.from_numpy(outputs[f"{name}_low_rank_lm_head"]),
                               rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(m.logits_from_hidden(hidden), torch.from_numpy(outputs[f"{name}_logits"]),
                               rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m.advance(tokens, hidden), torch.from_numpy(outputs[f"{name}_advance"]),
                               rtol=1e-5, atol=1e-6)
    assert m.init_empty_hidden(3, device=torch.device("cpu")).shape == tuple(outputs[f"{name}_empty_hidden"].shape)


@pytest.mark.parametrize("name", ["markov_merged", "markov_factorized"])
def test_markov_head_matches_reference(name, expected, outputs, target):
    rec = expected[name]
    m = D.MarkovDeLSLocalHead.from_checkpoint(checkpoint_path=str(CKPT / f"{name}.pt"), target_model=target,
                                              dtype=torch.float32, device=torch.device("cpu"))
    assert (m.vocab_size, m.rank) == (rec["vocab_size"], rec["rank"])
    torch.testing.assert_close(m.logits_from_token(torch.from_numpy(outputs["prev"])),
                               torch.from_numpy(outputs[f"{name}_logits"]), rtol=1e-5, atol=1e-6)


def test_position_mix_head_matches_reference(expected, outputs, target):
    rec = expected["position_mix"]
    m = D.PositionMixJointHead.from_checkpoint(checkpoint_path=str(CKPT / "position_mix.pt"), target_model=target,
                                               block_size=16, dtype=torch.float32, device=torch.device("cpu"))
    a, b = m.alpha_beta_schedules()
    np.testing.assert_allclose(a, rec["alpha"], rtol=1e-6)
    np.testing.assert_allclose(b, rec["beta"], rtol=1e-6)
    assert m.shift_label == rec["shift_label"] and m.pure_draft_prefix_len == rec["pure"]
    hidden = torch.from_numpy(outputs["hidden"])
    np.testing.assert_allclose(m.baseline_logits.numpy(), outputs["position_mix_baseline"], rtol=1e-6)
    torch.testing.assert_close(m.logits_from_hidden(hidden), torch.from_numpy(outputs["position_mix_logits"]),
                               rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m.advance(torch.from_numpy(outputs["tokens"]), hidden),
                               torch.from_numpy(outputs["position_mix_advance"]), rtol=1e-5, atol=1e-6)


def test_local_head_constructor_errors(target):
    with pytest.raises(ValueError, match="rank_activation"):
        D.DeLSLocalHead(target_model=target, vocab_size=64, embed_dim=8, gru_hidden_dim=16, low_rank_dim=4,
                        lm_head_mode="low_rank", rank_activation="relu", dtype=torch.float32, device="cpu")
    with pytest.raises(ValueError, match="target_lm_head is required"):
        D.DeLSLocalHead(target_model=target, vocab_size=64, embed_dim=8, gru_hidden_dim=16, low_rank_dim=4,
                        lm_head_mode="target_lm_head", dtype=torch.float32, device="cpu")
    with pytest.raises(ValueError, match="rank-2"):
        D.MarkovDeLSLocalHead(embedding_weight=torch.zeros(3), lm_head_weight=torch.zeros(3, 2),
                              dtype=torch.float32, device="cpu")
    with pytest.raises(ValueError, match="rank mismatch"):
        D.MarkovDeLSLocalHead(embedding_weight=torch.zeros(3, 4), lm_head_weight=torch.zeros(3, 2),
                              dtype=torch.float32, device="cpu")
    with tempfile.TemporaryDirectory() as td:
        torch.save({"model_config": {}}, Path(td) / "x.pt")
        with pytest.raises(ValueError, match="model_config and model_state_dict"):
            D.DeLSLocalHead.from_checkpoint(checkpoint_path=str(Path(td) / "x.pt"), target_model=target,
                                            dtype=torch.float32, device="cpu")
