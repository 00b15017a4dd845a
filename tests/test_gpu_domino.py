"""The drop-in Domino correction runner (kernel/domino.py) and its two new entry points
(dels_linear_bf16, dels_correction_mid_bf16) against the oracle and the reference's own
runner outputs (tests/golden/domino.npz: its torch path in fp32 / bf16 and its fused
Triton step).  Needs a B200.  Token comparisons stop at the first step whose exact top-2
gap is below the tolerance (after a legitimate near-tie greedy rollouts may part ways)."""

from __future__ import annotations

import json
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import dels_oracle as O

pytestmark = pytest.mark.gpu


class _Draft(nn.Module):
    def __init__(self, H, G, M, V, bias, middle=None):
        super().__init__()
        self.prefix_gru = nn.GRU(input_size=H, hidden_size=G, num_layers=1, batch_first=True, bias=bias)
        self.embed_proj = nn.Sequential(nn.Linear(H + G, M, bias=bias), middle or nn.SiLU(),
                                        nn.Linear(M, V, bias=bias))


def _target(embed, dev):
    V, H = embed.shape
    t = types.SimpleNamespace(model=types.SimpleNamespace(embed_tokens=nn.Embedding(V, H)))
    with torch.no_grad():
        t.model.embed_tokens.weight.copy_(torch.from_numpy(np.asarray(embed)))
    t.model.embed_tokens = t.model.embed_tokens.to(device=dev, dtype=torch.bfloat16)
    return t


def _compare(ours, gaps, ref, thresh):
    n = 0
    for b in range(ours.shape[0]):
        for t in range(ours.shape[1]):
            if gaps[b, t] <= thresh:
                break
            assert ours[b, t] == ref[b, t], (b, t, ours[b], ref[b])
            n += 1
    return n


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def test_linear_bf16_matches_oracle(cuda_device):
    from dels_b200 import ops

    rng = np.random.default_rng(31)
    for rows, K, N, bias in ((7, 96, 40, True), (300, 520, 200, False), (1, 64, 24, True)):
        x = O.bf16_round(rng.standard_normal((rows, K)).astype(np.float32))
        w = O.bf16_round((rng.standard_normal((N, K)) * 0.1).astype(np.float32))
        b = O.bf16_round(rng.standard_normal(N).astype(np.float32)) if bias else None
        out = ops.linear_bf16(_bf16(x, cuda_device), _bf16(w, cuda_device),
                              _bf16(b, cuda_device) if bias else None).float().cpu().numpy()
        acc = x.astype(np.float64) @ w.astype(np.float64).T + (0.0 if b is None else b.astype(np.float64))
        ref = O.bf16_round(acc.astype(np.float32))
        assert np.mean(out == ref) > 0.99  # one rounding of an fp32 accumulation
        np.testing.assert_allclose(out, ref, rtol=2 ** -7, atol=1e-3)


def test_linear_bf16_single_split_epilogue(cuda_device):
    """Vocabulary-sized N: the output tiles fill the device, K is not split and the GEMM's
    epilogue writes bf16 itself (no partials, workspace = header).  16-byte stores (packed
    rows) and element stores (a row stride that is not a multiple of 8) must give the
    same bits, within one bf16 rounding of the exact sum."""
    from dels_b200 import ops

    rng = np.random.default_rng(33)
    # 14 rows: one 128-row tile (single-CTA kernel); 130 and 300 rows: CTA-pair tiles
    for rows, K, N, bias in ((14, 512, 40000, True), (130, 256, 38000, False), (300, 256, 38000, True)):
        assert ops.linear_workspace_bytes(rows, K, N) == ops.linear_workspace_bytes(0, K, N)
        x = O.bf16_round(rng.standard_normal((rows, K)).astype(np.float32))
        w = O.bf16_round((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
        b = O.bf16_round(rng.standard_normal(N).astype(np.float32)) if bias else None
        xt, wt = _bf16(x, cuda_device), _bf16(w, cuda_device)
        bt = _bf16(b, cuda_device) if bias else None
        packed = ops.linear_bf16(xt, wt, bt)
        wide = torch.full((rows, N + 3), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        strided = ops.linear_bf16(xt, wt, bt, out=wide[:, :N])
        assert torch.equal(packed.view(torch.int16), strided.view(torch.int16))
        assert torch.isnan(wide[:, N:].float()).all()  # nothing written past N
        out = packed.float().cpu().numpy()
        acc = x.astype(np.float64) @ w.astype(np.float64).T + (0.0 if b is None else b.astype(np.float64))
        ref = O.bf16_round(acc.astype(np.float32))
        assert np.mean(out == ref) > 0.99
        np.testing.assert_allclose(out, ref, rtol=2 ** -7, atol=1e-3)


def test_correction_mid_matches_oracle(cuda_device):
    from dels_b200 import ops

    rng = np.random.default_rng(32)
    B, G, M, S = 5, 64, 48, 3
    h = O.bf16_round(rng.standard_normal((B, G)).astype(np.float32))
    w_s = O.bf16_round((rng.standard_normal((M, G)) * 0.2).astype(np.float32))
    z = O.bf16_round(rng.standard_normal((B, S, M)).astype(np.float32))
    alpha = 0.7
    dev = cuda_device
    z_t = _bf16(z, dev)
    out = torch.empty(B, M, dtype=torch.bfloat16, device=dev)
    keys = torch.zeros(B, dtype=torch.int64, device=dev)
    ops.correction_mid(_bf16(h, dev), _bf16(w_s, dev), z_t[:, 1, :], torch.tensor([alpha], device=dev), out,
                       keys=keys)
    s = O.bf16_round((h.astype(np.float64) @ w_s.astype(np.float64).T).astype(np.float32)).astype(np.float64)
    pre = z[:, 1, :].astype(np.float64) + s
    ref = O.bf16_round((alpha * pre / (1.0 + np.exp(-pre))).astype(np.float32))
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=2 ** -7, atol=1e-6)
    assert (keys.cpu().numpy() == np.iinfo(np.int64).min).all()


def test_correction_mid_tc_matches_oracle(cuda_device):
    """The tensor-core variant (split-K W_s h, then the SiLU epilogue) at 40 rows."""
    from dels_b200 import ops

    rng = np.random.default_rng(33)
    B, G, M = 40, 64, 48
    h = O.bf16_round(rng.standard_normal((B, G)).astype(np.float32))
    w_s = O.bf16_round((rng.standard_normal((M, G)) * 0.2).astype(np.float32))
    z = O.bf16_round(rng.standard_normal((B, M)).astype(np.float32))
    alpha = 0.6
    dev = cuda_device
    out = torch.empty(B, M, dtype=torch.bfloat16, device=dev)
    keys = torch.zeros(B, dtype=torch.int64, device=dev)
    ws = ops.Workspace(ops.correction_mid_tc_workspace_bytes(B, G, M), dev)
    ops.correction_mid_tc(_bf16(h, dev), _bf16(w_s, dev), _bf16(z, dev), torch.tensor([alpha], device=dev), out,
                          keys=keys, ws=ws)
    s = O.bf16_round((h.astype(np.float64) @ w_s.astype(np.float64).T).astype(np.float32)).astype(np.float64)
    pre = z.astype(np.float64) + s
    ref = O.bf16_round((alpha * pre / (1.0 + np.exp(-pre))).astype(np.float32))
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=2 ** -7, atol=1e-6)
    assert (keys.cpu().numpy() == np.iinfo(np.int64).min).all()


@pytest.mark.parametrize("overlap", ["1", "split", "0"])
def test_domino_runner_matches_reference_fixture(cuda_device, golden_dir, monkeypatch, overlap):
    """The three small-batch schedules: the GRU gates fused into the correction layer or a
    gates kernel before it, both with the next W_hh h on the scorer's helper warps, and the
    GRU step kernel first."""
    from kernel.domino import DraftCorrectionGraphRunner

    monkeypatch.setenv("DELS_RUNNER_OVERLAP_ROWS", "4" if overlap == "1" else "0")
    monkeypatch.setenv("DELS_RUNNER_SPLIT_GRU", "0" if overlap == "0" else "1")
    g = np.load(golden_dir / "domino.npz")
    total = 0
    for c in json.loads(str(g["meta"])):
        n = c["name"]
        draft = _Draft(c["H"], c["G"], c["M"], c["V"], c["bias"])
        with torch.no_grad():
            for k, prm in draft.named_parameters():
                prm.copy_(torch.from_numpy(g[f"{n}_{k.replace('.', '_')}"]))
        draft = draft.to(device=cuda_device, dtype=torch.bfloat16)
        runner = DraftCorrectionGraphRunner(
            draft_model=draft, target_model=_target(g[f"{n}_embed"], cuda_device), batch_size=c["B"],
            steps=c["steps"], hidden_dim=c["H"], gru_hidden_dim=c["G"], vocab_size=c["V"],
            prefix_token_count=c["P"], device=cuda_device, guidance_alpha=c["alpha"],
        )
        assert runner._can_triton_fuse
        out = runner(torch.from_numpy(g[f"{n}_prefix"]).to(cuda_device), _bf16(g[f"{n}_hiddens"], cuda_device),
                     _bf16(g[f"{n}_base"], cuda_device), c["alpha"]).cpu().numpy()
        assert out.shape == (c["B"], c["steps"]) and out.dtype == np.int64
        opt = (lambda k: g[f"{n}_{k}"]) if c["bias"] else (lambda k: None)
        toks, gaps = O.domino_runner_rollout(
            g[f"{n}_prefix"], g[f"{n}_hiddens"], g[f"{n}_base"], alpha=c["alpha"], bf16=True,
            embed=g[f"{n}_embed"], w_ih=g[f"{n}_prefix_gru_weight_ih_l0"], w_hh=g[f"{n}_prefix_gru_weight_hh_l0"],
            b_ih=opt("prefix_gru_bias_ih_l0"), b_hh=opt("prefix_gru_bias_hh_l0"),
            w1=g[f"{n}_embed_proj_0_weight"], b1=opt("embed_proj_0_bias"), fc2=g[f"{n}_embed_proj_2_weight"],
            b2=opt("embed_proj_2_bias"),
        )
        total += _compare(out, gaps, toks, 1e-2)
        _compare(out, gaps, g[f"{n}_tokens_bf16_fused"], 0.05)
        _compare(out, gaps, g[f"{n}_tokens_bf16"], 0.05)
    assert total >= 12


def test_domino_runner_validation_errors(cuda_device):
    from kernel.domino import DraftCorrectionGraphRunner, unwrap_correction_mlp

    with pytest.raises(TypeError, match="nn.Sequential"):
        unwrap_correction_mlp(nn.Linear(4, 4))
    with pytest.raises(ValueError, match="at least two layers"):
        unwrap_correction_mlp(nn.Sequential(nn.Linear(4, 4)))
    with pytest.raises(ValueError, match="first layer"):
        unwrap_correction_mlp(nn.Sequential(nn.SiLU(), nn.Linear(4, 4)))
    with pytest.raises(ValueError, match="last layer"):
        unwrap_correction_mlp(nn.Sequential(nn.Linear(4, 4), nn.SiLU()))
    embed = O.bf16_round(np.random.default_rng(0).standard_normal((64, 16)).astype(np.float32))
    kw = dict(target_model=_target(embed, cuda_device), batch_size=1, steps=2, hidden_dim=16, gru_hidden_dim=8,
              vocab_size=64, prefix_token_count=1, device=cuda_device)
    with pytest.raises(ValueError, match="input dim mismatch"):
        DraftCorrectionGraphRunner(draft_model=_Draft(16, 8, 12, 64, False).to(cuda_device, torch.bfloat16),
                                   **{**kw, "gru_hidden_dim": 4})
    with pytest.raises(ValueError, match="SiLU"):
        DraftCorrectionGraphRunner(draft_model=_Draft(16, 8, 12, 64, False, nn.ReLU()).to(cuda_device, torch.bfloat16),
                                   **kw)
    with pytest.raises(ValueError, match="bf16"):
        DraftCorrectionGraphRunner(draft_model=_Draft(16, 8, 12, 64, False).to(cuda_device), **kw)
    runner = DraftCorrectionGraphRunner(draft_model=_Draft(16, 8, 12, 64, False).to(cuda_device, torch.bfloat16),
                                        guidance_alpha=0.5, **kw)
    with pytest.raises(ValueError, match="fixed domino guidance alpha"):
        runner(torch.zeros(1, 1, dtype=torch.long, device=cuda_device),
               torch.zeros(1, 2, 16, dtype=torch.bfloat16, device=cuda_device),
               torch.zeros(1, 2, 64, dtype=torch.bfloat16, device=cuda_device), 0.25)


def test_domino_runner_full_vocab(cuda_device):
    """Full vocabulary (151936), batch 2, 8 steps, 2 prefix tokens, against the oracle."""
    from kernel.domino import DraftCorrectionGraphRunner

    V, H, G, M, B, S, P, alpha = 151936, 1024, 512, 512, 2, 8, 2, 1.0
    gen = torch.Generator(device="cpu").manual_seed(41)
    draft = _Draft(H, G, M, V, False)
    with torch.no_grad():
        for prm in draft.parameters():
            prm.copy_((torch.randn(prm.shape, generator=gen) * 0.05).to(torch.bfloat16).float())
    embed = (torch.randn(V, H, generator=gen) * 0.5).to(torch.bfloat16).float().numpy()
    hiddens = (torch.randn(B, S, H, generator=gen)).to(torch.bfloat16).float().numpy()
    base = (torch.randn(B, S, V, generator=gen)).to(torch.bfloat16).float().numpy()
    prefix = torch.randint(0, V, (B, P), generator=gen).numpy()
    params = {k.replace(".", "_"): p.detach().numpy().copy() for k, p in draft.named_parameters()}
    runner = DraftCorrectionGraphRunner(
        draft_model=draft.to(cuda_device, torch.bfloat16), target_model=_target(embed, cuda_device), batch_size=B,
        steps=S, hidden_dim=H, gru_hidden_dim=G, vocab_size=V, prefix_token_count=P, device=cuda_device,
        guidance_alpha=alpha,
    )
    out = runner(torch.from_numpy(prefix).to(cuda_device), _bf16(hiddens, cuda_device),
                 _bf16(base, cuda_device)).cpu().numpy()
    toks, gaps = O.domino_runner_rollout(
        prefix, hiddens, base, alpha=alpha, bf16=True, embed=embed, w_ih=params["prefix_gru_weight_ih_l0"],
        w_hh=params["prefix_gru_weight_hh_l0"], b_ih=None, b_hh=None, w1=params["embed_proj_0_weight"], b1=None,
        fc2=params["embed_proj_2_weight"], b2=None,
    )
    assert _compare(out, gaps, toks, 1e-2) >= 4


def test_domino_runner_batch20_with_biases(cuda_device):
    """20 rows (the tensor-core W_hh product, then the gates) with every bias present, including
    the GRU's b_hh on the zero first state, against the oracle."""
    from kernel.domino import DraftCorrectionGraphRunner

    V, H, G, M, B, S, P, alpha = 3001, 64, 48, 40, 20, 4, 2, 0.8
    gen = torch.Generator(device="cpu").manual_seed(43)
    draft = _Draft(H, G, M, V, True)
    with torch.no_grad():
        for prm in draft.parameters():
            prm.copy_((torch.randn(prm.shape, generator=gen) * 0.2).to(torch.bfloat16).float())
    embed = (torch.randn(V, H, generator=gen) * 0.5).to(torch.bfloat16).float().numpy()
    hiddens = (torch.randn(B, S, H, generator=gen)).to(torch.bfloat16).float().numpy()
    base = (torch.randn(B, S, V, generator=gen)).to(torch.bfloat16).float().numpy()
    prefix = torch.randint(0, V, (B, P), generator=gen).numpy()
    prm = {k.replace(".", "_"): p.detach().numpy().copy() for k, p in draft.named_parameters()}
    runner = DraftCorrectionGraphRunner(
        draft_model=draft.to(cuda_device, torch.bfloat16), target_model=_target(embed, cuda_device), batch_size=B,
        steps=S, hidden_dim=H, gru_hidden_dim=G, vocab_size=V, prefix_token_count=P, device=cuda_device,
        guidance_alpha=alpha,
    )
    assert runner._tc
    out = runner(torch.from_numpy(prefix).to(cuda_device), _bf16(hiddens, cuda_device),
                 _bf16(base, cuda_device)).cpu().numpy()
    toks, gaps = O.domino_runner_rollout(
        prefix, hiddens, base, alpha=alpha, bf16=True, embed=embed, w_ih=prm["prefix_gru_weight_ih_l0"],
        w_hh=prm["prefix_gru_weight_hh_l0"], b_ih=prm["prefix_gru_bias_ih_l0"], b_hh=prm["prefix_gru_bias_hh_l0"],
        w1=prm["embed_proj_0_weight"], b1=prm["embed_proj_0_bias"], fc2=prm["embed_proj_2_weight"],
        b2=prm["embed_proj_2_bias"],
    )
    assert _compare(out, gaps, toks, 1e-2) >= B * S // 2


@pytest.mark.parametrize("B", [6, 8])
def test_domino_runner_split_schedule_5_to_8_rows(cuda_device, B):
    """5-8 rows: the gates kernel, the correction layer and the scorer whose helper warps
    (built for 8 rows) compute the next W_hh h, every bias present, against the oracle."""
    from kernel.domino import DraftCorrectionGraphRunner

    V, H, G, M, S, P, alpha = 3001, 64, 48, 40, 4, 2, 0.8
    gen = torch.Generator(device="cpu").manual_seed(47 + B)
    draft = _Draft(H, G, M, V, True)
    with torch.no_grad():
        for prm in draft.parameters():
            prm.copy_((torch.randn(prm.shape, generator=gen) * 0.2).to(torch.bfloat16).float())
    embed = (torch.randn(V, H, generator=gen) * 0.5).to(torch.bfloat16).float().numpy()
    hiddens = (torch.randn(B, S, H, generator=gen)).to(torch.bfloat16).float().numpy()
    base = (torch.randn(B, S, V, generator=gen)).to(torch.bfloat16).float().numpy()
    prefix = torch.randint(0, V, (B, P), generator=gen).numpy()
    prm = {k.replace(".", "_"): p.detach().numpy().copy() for k, p in draft.named_parameters()}
    runner = DraftCorrectionGraphRunner(
        draft_model=draft.to(cuda_device, torch.bfloat16), target_model=_target(embed, cuda_device), batch_size=B,
        steps=S, hidden_dim=H, gru_hidden_dim=G, vocab_size=V, prefix_token_count=P, device=cuda_device,
        guidance_alpha=alpha,
    )
    assert runner._split_gru and runner._keys_only and not runner._tc
    out = runner(torch.from_numpy(prefix).to(cuda_device), _bf16(hiddens, cuda_device),
                 _bf16(base, cuda_device)).cpu().numpy()
    toks, gaps = O.domino_runner_rollout(
        prefix, hiddens, base, alpha=alpha, bf16=True, embed=embed, w_ih=prm["prefix_gru_weight_ih_l0"],
        w_hh=prm["prefix_gru_weight_hh_l0"], b_ih=prm["prefix_gru_bias_ih_l0"], b_hh=prm["prefix_gru_bias_hh_l0"],
        w1=prm["embed_proj_0_weight"], b1=prm["embed_proj_0_bias"], fc2=prm["embed_proj_2_weight"],
        b2=prm["embed_proj_2_bias"],
    )
    assert _compare(out, gaps, toks, 1e-2) >= B * S // 2
