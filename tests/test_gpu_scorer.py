"""Parity of the CUDA scorers with the oracle / reference fixtures (needs a B200).

Tolerances (from the path's contract): bf16 workloads — scores within 1e-2 absolute,
tokens identical on every row whose exact top-2 gap exceeds 1e-2; fp32 workloads —
scores within 1e-5, tokens identical where the gap exceeds 1e-5.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import dels_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
F32_TOL = 1e-5


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def _f32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _check_tokens(tokens, best_scores, ref_scores, tol):
    """tokens / winning scores of the kernel against exact reference scores."""
    tokens = np.asarray(tokens)
    ref_scores = np.asarray(ref_scores, dtype=np.float64)
    ref_tok = O.argmax_first(ref_scores)
    gap = O.top2_gap(ref_scores)
    rows = np.arange(len(tokens))
    ref_best = ref_scores[rows, ref_tok]
    # The chosen token's exact score is within tol of the best, and the reported score
    # is within tol of that exact score.
    assert np.all(ref_scores[rows, tokens] >= ref_best - tol), "kernel picked a clearly worse token"
    if best_scores is not None:
        np.testing.assert_allclose(best_scores, ref_scores[rows, tokens], rtol=0, atol=tol)
    clear = gap > tol
    np.testing.assert_array_equal(tokens[clear], ref_tok[clear])
    return clear.mean()


def _rand_case(rng, rows, H, r, V, n_pos):
    h = O.bf16_round(rng.standard_normal((rows, H)).astype(np.float32))
    W = O.bf16_round((rng.standard_normal((V, H)) * 0.02).astype(np.float32))
    Ut = O.bf16_round((rng.standard_normal((r, H)) * 0.02).astype(np.float32))
    Vr = O.bf16_round((rng.standard_normal((V, r)) * 0.02).astype(np.float32))
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = np.linspace(0.5, 0.1, n_pos)
    beta = np.linspace(0.3, 0.0, n_pos)
    return h, W, Ut, Vr, prior, alpha, beta


SHAPES = [
    # rows, H, r, V, n_pos, activation, prior
    # at most 32 rows: the skinny scorer (16- or 32-column row tiles)
    (16, 256, 64, 4099, 16, "identity", True),
    (1, 128, 64, 1000, 1, "identity", True),
    (24, 256, 64, 5003, 8, "silu", True),
    # at most 4 rows with a long K (17 K blocks) over 157 vocabulary tiles on 148 CTAs:
    # a partial last wave and a partial last tile
    (1, 1024, 64, 20000, 1, "identity", True),
    (3, 1024, 64, 20000, 4, "silu", True),
    # 33..128 rows: one 128-row tile; more: CTA pairs
    (48, 320, 96, 2347, 16, "identity", True),
    (130, 320, 96, 2347, 8, "silu", True),
    (300, 200, 40, 517, 16, "identity", False),
    (512, 4096, 256, 3000, 16, "identity", True),
]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"r{s[0]}_H{s[1]}_r{s[2]}_V{s[3]}" for s in SHAPES])
def test_draft_score_bf16_matches_oracle(cuda_device, shape):
    from dels_b200 import ops

    rows, H, r, V, n_pos, act, with_prior = shape
    rng = np.random.default_rng(rows * 7 + V)
    h, W, Ut, Vr, prior, alpha, beta = _rand_case(rng, rows, H, r, V, n_pos)
    dev = cuda_device
    out = ops.draft_score_bf16(
        _bf16(h, dev), _bf16(W, dev), _bf16(Ut, dev), _bf16(Vr, dev), _f32(prior, dev) if with_prior else None,
        _f32(alpha, dev), _f32(beta, dev), n_pos=n_pos, activation=act, with_scores=True,
    )
    torch.cuda.synchronize()
    tok, sc, gap = O.draft_score_bf16(h, W, Ut, Vr, prior if with_prior else None, alpha, beta, n_pos=n_pos,
                                      activation=act)
    frac = _check_tokens(out.tokens.cpu().numpy(), out.scores.cpu().numpy(), sc, BF16_TOL)
    assert frac > 0.5
    # the packed keys decode to the same tokens
    np.testing.assert_array_equal(O.key_index(out.keys.cpu().numpy()), out.tokens.cpu().numpy())


def test_rank_projection_matches_oracle(cuda_device):
    from dels_b200 import ops

    rng = np.random.default_rng(5)
    rows, K, r = 200, 1000, 72
    x = O.bf16_round(rng.standard_normal((rows, K)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal((r, K)) * 0.05).astype(np.float32))
    alpha = np.linspace(0.9, 0.2, 7)
    for act in ("identity", "silu"):
        s, ss = ops.rank_project_bf16(_bf16(x, cuda_device), _bf16(w, cuda_device), _f32(alpha, cuda_device),
                                      n_pos=7, activation=act)
        ref = O.rank_state_bf16(x, w, act)
        got = s.float().cpu().numpy()
        # bf16 rounding of an fp32 accumulation: equal except at rounding boundaries
        assert np.mean(got == ref) > 0.99
        np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-3)
        pos = np.arange(rows) % 7
        ref_scaled = O.bf16_round((alpha[pos][:, None].astype(np.float32) * got).astype(np.float32))
        np.testing.assert_array_equal(ss.float().cpu().numpy(), ref_scaled)


def test_base_variant_matches_oracle(cuda_device):
    """The DeLSGraphRunner step: base logits + alpha * low-rank - beta * prior."""
    from dels_b200 import ops

    for rows in (5, 24, 40, 150):  # skinny (16 / 32 columns), one 128-row tile, CTA pairs
        _base_variant_case(cuda_device, rows)


def _base_variant_case(dev, rows):
    from dels_b200 import ops

    rng = np.random.default_rng(9 + rows)
    r, V, n_pos = 48, 3001, 5
    base = O.bf16_round(rng.standard_normal((rows, V)).astype(np.float32))
    s = O.bf16_round(rng.standard_normal((rows, r)).astype(np.float32))
    Vr = O.bf16_round((rng.standard_normal((V, r)) * 0.1).astype(np.float32))
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = np.linspace(0.8, 0.3, n_pos)
    beta = np.linspace(0.1, 0.3, n_pos)
    s_scaled = O.bf16_round((alpha[np.arange(rows) % n_pos][:, None] * s).astype(np.float32))
    for ld_extra in (7, 3):  # row stride 3008 takes the 16-byte vector path, 3004 the scalar one
        base_t = torch.zeros(rows, V + ld_extra, dtype=torch.bfloat16, device=dev)
        base_t[:, :V] = _bf16(base, dev)
        out = ops.fused_argmax_base_bf16(base_t[:, :V], _bf16(s_scaled, dev), _bf16(Vr, dev), _f32(prior, dev),
                                         _f32(beta, dev), n_pos=n_pos, with_scores=True)
        torch.cuda.synchronize()
        ref = O.base_scores(base, s_scaled, Vr, prior, np.ones(rows), beta[np.arange(rows) % n_pos])
        _check_tokens(out.tokens.cpu().numpy(), out.scores.cpu().numpy(), ref, BF16_TOL)


def test_scorer_matches_reference_fixtures(cuda_device, golden_dir):
    """Reference outputs (tests/golden/scorer.npz) through the CUDA bf16 scorer."""
    from dels_b200 import ops

    g = np.load(golden_dir / "scorer.npz")
    for c in json.loads(str(g["meta"])):
        n = c["name"]
        prior = g[f"{n}_prior_bf16"] if c["prior"] else None
        dev = cuda_device
        out = ops.draft_score_bf16(
            _bf16(g[f"{n}_h"], dev), _bf16(g[f"{n}_W"], dev), _bf16(g[f"{n}_Ut"], dev), _bf16(g[f"{n}_Vr"], dev),
            None if prior is None else _f32(prior, dev), _f32(g[f"{n}_alpha"], dev), _f32(g[f"{n}_beta"], dev),
            n_pos=c["P"], activation=c["activation"], with_scores=True,
        )
        tok, sc, gap = O.draft_score_bf16(g[f"{n}_h"], g[f"{n}_W"], g[f"{n}_Ut"], g[f"{n}_Vr"], prior,
                                          g[f"{n}_alpha"], g[f"{n}_beta"], n_pos=c["P"], activation=c["activation"])
        got = out.tokens.cpu().numpy()
        # against the reference's own bf16 tokens wherever the exact gap is clear of
        # the reference's bf16 rounding
        clear = gap > 0.05
        np.testing.assert_array_equal(got[clear], g[f"{n}_tokens_bf16"][clear])
        _check_tokens(got, out.scores.cpu().numpy(), sc, BF16_TOL)


def test_draft_score_f32_matches_oracle(cuda_device, golden_dir):
    from dels_b200 import ops

    rng = np.random.default_rng(1)
    for rows, H, r, V, n_pos in ((16, 256, 64, 3001, 1), (5, 64, 8, 999, 5), (40, 128, 16, 2000, 16)):
        h = rng.standard_normal((rows, H)).astype(np.float32)
        W = (rng.standard_normal((V, H)) * 0.02).astype(np.float32)
        Ut = (rng.standard_normal((r, H)) * 0.02).astype(np.float32)
        Vr = (rng.standard_normal((V, r)) * 0.02).astype(np.float32)
        prior = O.zipf_log_prior(V).astype(np.float32)
        alpha = np.linspace(0.3, 0.6, n_pos)
        beta = np.linspace(0.3, 0.1, n_pos)
        dev = cuda_device
        out = ops.draft_score_f32(_f32(h, dev), _f32(W, dev), _f32(Ut, dev), _f32(Vr, dev), _f32(prior, dev),
                                  _f32(alpha, dev), _f32(beta, dev), n_pos=n_pos, with_scores=True)
        tok, sc, gap = O.draft_score_f32(h, W, Ut, Vr, prior, alpha, beta, n_pos=n_pos)
        _check_tokens(out.tokens.cpu().numpy(), out.scores.cpu().numpy(), sc, F32_TOL)
    # the reference's fp32 fixtures (identity activation cases)
    g = np.load(golden_dir / "scorer.npz")
    for c in json.loads(str(g["meta"])):
        if c["activation"] != "identity" or c["H"] % 4 or c["r"] % 4:
            continue
        n = c["name"]
        prior = g[f"{n}_prior_f32"] if c["prior"] else None
        out = ops.draft_score_f32(
            _f32(g[f"{n}_h"], dev), _f32(g[f"{n}_W"], dev), _f32(g[f"{n}_Ut"], dev), _f32(g[f"{n}_Vr"], dev),
            None if prior is None else _f32(prior, dev), _f32(g[f"{n}_alpha"], dev), _f32(g[f"{n}_beta"], dev),
            n_pos=c["P"], with_scores=True,
        )
        _check_tokens(out.tokens.cpu().numpy(), out.scores.cpu().numpy(), g[f"{n}_final_f32"], F32_TOL)


@pytest.mark.parametrize("rows", [3, 40, 150], ids=["skinny", "tile", "pair"])
def test_edge_cases(cuda_device, rows):
    from dels_b200 import ops, _lib

    dev = cuda_device
    # all-equal scores: lowest index wins
    H, r, V = 64, 64, 5000
    h = torch.zeros(rows, H, dtype=torch.bfloat16, device=dev)
    W = torch.zeros(V, H, dtype=torch.bfloat16, device=dev)
    Ut = torch.zeros(r, H, dtype=torch.bfloat16, device=dev)
    Vr = torch.zeros(V, r, dtype=torch.bfloat16, device=dev)
    a = torch.ones(1, device=dev)
    out = ops.draft_score_bf16(h, W, Ut, Vr, None, a, a, with_scores=True)
    assert out.tokens.tolist() == [0] * rows
    # planted ties in vocabulary tiles owned by different CTAs: the lower index wins
    W2 = torch.zeros(V, H, dtype=torch.bfloat16, device=dev)
    W2[4700, 0] = 1.0
    W2[3001, 0] = 1.0
    W2[5, 0] = 0.5
    h2 = torch.zeros(rows, H, dtype=torch.bfloat16, device=dev)
    h2[:, 0] = 1.0
    out = ops.draft_score_bf16(h2, W2, Ut, Vr, None, a, a, with_scores=True)
    assert out.tokens.tolist() == [3001] * rows
    assert out.scores.tolist() == [1.0] * rows
    # NaN scores win, and the first NaN index among them (torch.argmax)
    W3 = W2.clone()
    W3[4100, 1] = float("nan")
    W3[3900, 1] = float("nan")
    h3 = h2.clone()
    h3[:, 1] = 1.0
    out = ops.draft_score_bf16(h3, W3, Ut, Vr, None, a, a, with_scores=True)
    assert out.tokens.tolist() == [3900] * rows
    assert torch.isnan(out.scores).all()
    # a prior of -inf everywhere but one token (beta < 0 makes it +inf there)
    prior = torch.full((V,), 0.0, device=dev)
    prior[613] = -1.0
    out = ops.draft_score_bf16(h2, W2, Ut, Vr, prior, a, torch.full((1,), 5.0, device=dev), with_scores=True)
    assert out.tokens.tolist() == [613] * rows
    # zero rows is a no-op
    e = ops.draft_score_bf16(h2[:0], W2, Ut, Vr, None, a, a)
    assert e.tokens.numel() == 0
    # argument errors are ValueErrors raised before any launch
    with pytest.raises(ValueError):
        ops.draft_score_bf16(h2, W2[:, :32], Ut, Vr, None, a, a)
    with pytest.raises(_lib.DelsArgumentError):
        ops.draft_score_bf16(h2[:, 1:], W2[:, 1:], Ut[:, 1:], Vr, None, a, a)  # misaligned rows
    torch.cuda.synchronize()


@pytest.mark.parametrize("rows", [3, 40, 150, 300], ids=["skinny", "tile", "pair", "pair2"])
def test_integer_score_ties(cuda_device, rows):
    """Scores that are small integers, so most rows have their maximum at many columns spread
    over chunks, tiles and CTAs: the token must be the first of them exactly (torch.argmax).
    V = 5003 leaves a partial last chunk and tile."""
    from dels_b200 import ops

    dev = cuda_device
    g = torch.Generator(device="cpu").manual_seed(11)
    H, r, V = 64, 64, 5003
    h = (torch.rand(rows, H, generator=g) < 0.15).float()
    W = torch.randint(-1, 2, (V, H), generator=g).float()
    prior = torch.randint(0, 2, (V,), generator=g).float()
    Ut = torch.zeros(r, H)
    Vr = torch.randint(-1, 2, (V, r), generator=g).float()
    ref = h.double() @ W.double().T - prior.double()[None, :]  # exact: small integers
    expect = ref.argmax(dim=1)
    assert ((ref == ref.max(dim=1, keepdim=True).values).sum(dim=1) > 1).float().mean() > 0.5  # ties are common
    bf = lambda t: t.to(dev, torch.bfloat16)  # noqa: E731
    one = torch.ones(1, device=dev)
    out = ops.draft_score_bf16(bf(h), bf(W), bf(Ut), bf(Vr), prior.to(dev), one, one, with_scores=True)
    assert out.tokens.cpu().tolist() == expect.tolist()
    assert out.scores.cpu().double().tolist() == ref.max(dim=1).values.tolist()


def test_keys_only_vocab_shards_combine(cuda_device):
    """Vocab-sharded scoring emulated on one GPU: per-slice keys + max = full result."""
    from dels_b200 import ops, workloads

    dev = cuda_device
    rows, H, r, V = 64, 512, 64, 10007
    rng = np.random.default_rng(3)
    h, W, Ut, Vr, prior, alpha, beta = _rand_case(rng, rows, H, r, V, 16)
    full = ops.draft_score_bf16(_bf16(h, dev), _bf16(W, dev), _bf16(Ut, dev), _bf16(Vr, dev), _f32(prior, dev),
                                _f32(alpha, dev), _f32(beta, dev), n_pos=16, with_scores=True)
    for world in (2, 3, 8):
        keys = []
        for rank in range(world):
            v0, v1 = workloads.shard_range(V, world, rank)
            part = ops.draft_score_bf16(_bf16(h, dev), _bf16(W[v0:v1], dev), _bf16(Ut, dev), _bf16(Vr[v0:v1], dev),
                                        _f32(prior[v0:v1], dev), _f32(alpha, dev), _f32(beta, dev), n_pos=16,
                                        v_begin=v0, keys_only=True)
            keys.append(part.keys.clone())
        combined = torch.stack(keys).max(dim=0).values
        tok, sc = ops.keys_decode(combined)
        assert torch.equal(tok, full.tokens)
        assert torch.equal(sc, full.scores)


def test_workspace_status_clean(cuda_device):
    from dels_b200 import ops

    ws = ops.Workspace(1 << 22, cuda_device)
    rng = np.random.default_rng(0)
    h, W, Ut, Vr, prior, alpha, beta = _rand_case(rng, 8, 64, 16, 999, 8)
    dev = cuda_device
    for _ in range(3):
        ops.draft_score_bf16(_bf16(h, dev), _bf16(W, dev), _bf16(Ut, dev), _bf16(Vr, dev), _f32(prior, dev),
                             _f32(alpha, dev), _f32(beta, dev), n_pos=8, ws=ws)
    ws.check()
    assert int(ws.buf[0:4].view(torch.int32).item()) == 0  # completion counter left at zero
