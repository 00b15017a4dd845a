"""Parity of the acceptance / packing / RNN kernels and of the full-size workloads
(needs a B200).  Integer outputs are bit-exact; scores use the bf16 tolerance 1e-2."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import dels_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def _check(tokens, best, ref_scores, tol=BF16_TOL):
    from test_gpu_scorer import _check_tokens

    return _check_tokens(tokens, best, ref_scores, tol)


@pytest.mark.parametrize(
    "n_seq,P,V,commit_extra",
    [(256, 16, 151936, 0), (3, 40, 7, 1), (1500, 5, 3, 0), (1, 1, 2, 1), (0, 4, 10, 0), (64, 33, 2, 0)],
)
def test_accept_offsets_bit_exact(cuda_device, n_seq, P, V, commit_extra):
    from dels_b200 import ops

    rng = np.random.default_rng(n_seq + P)
    target = rng.integers(0, V, size=(n_seq, P + 1))
    draft = rng.integers(0, V, size=(n_seq, P))
    k = rng.integers(0, P + 1, size=n_seq)
    for b in range(n_seq):
        draft[b, : k[b]] = target[b, : k[b]]
    if n_seq > 2:
        draft[0] = target[0, :P]  # full acceptance
        draft[1, 0] = (target[1, 0] + 1) % max(V, 2)  # immediate rejection
    dev = cuda_device
    acc, off = ops.accept_offsets(torch.from_numpy(draft).to(dev), torch.from_numpy(target).to(dev),
                                  commit_extra=commit_extra)
    ref_acc, ref_off = O.accept_offsets(draft, target, commit_extra)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(off.cpu().numpy(), ref_off)


def test_accept_matches_reference_fixture(cuda_device, golden_dir):
    from dels_b200 import ops

    g = np.load(golden_dir / "accept.npz")
    dev = cuda_device
    acc, off = ops.accept_offsets(torch.from_numpy(g["verify"][:, 1:].copy()).to(dev),
                                  torch.from_numpy(g["posterior"]).to(dev))
    np.testing.assert_array_equal(acc.cpu().numpy(), g["accept"])


def test_pack_rows_bit_exact(cuda_device):
    from dels_b200 import ops

    rng = np.random.default_rng(4)
    n_seq, P, H = 37, 16, 136
    dev = cuda_device
    hidden = torch.randn(n_seq, P, H, device=dev).to(torch.bfloat16)
    accept = torch.from_numpy(rng.integers(0, P + 1, size=n_seq).astype(np.int32)).to(dev)
    offsets = torch.zeros(n_seq + 1, dtype=torch.int32, device=dev)
    offsets[1:] = torch.cumsum(accept, 0)
    packed, row_pos = ops.pack_rows(hidden, accept, offsets)
    ref, ref_pos = O.pack_rows(hidden.view(torch.int16).cpu().numpy(), accept.cpu().numpy(), offsets.cpu().numpy())
    total = int(offsets[-1])
    np.testing.assert_array_equal(packed[:total].view(torch.int16).cpu().numpy(), ref)
    np.testing.assert_array_equal(row_pos[:total].cpu().numpy(), ref_pos)


def test_ragged_pipeline_small(cuda_device):
    """Accept -> pack -> score with the device-side row count, against the oracle."""
    from dels_b200 import ops, workloads

    dev = cuda_device
    wl = workloads.cfg3(device=dev, V=5003, n_seq=40, P=16, H=256, r=64)
    t = wl.tensors
    acc, off = ops.accept_offsets(t["draft"], t["target"])
    packed, row_pos = ops.pack_rows(t["hidden"], acc, off)
    out = ops.draft_score_bf16(packed, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"],
                               n_pos=16, row_pos=row_pos, rows_dev=off[-1:], with_scores=True)
    torch.cuda.synchronize()
    total = int(off[-1])
    ref_acc, ref_off = O.accept_offsets(t["draft"].cpu().numpy(), t["target"].cpu().numpy())
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    tok, sc, gap = O.draft_score_bf16(f(packed[:total]), f(t["W"]), f(t["w_rank"]), f(t["Vr"]), f(t["prior"]),
                                      wl.alpha, wl.beta, n_pos=16, row_pos=row_pos[:total].cpu().numpy())
    _check(out.tokens[:total].cpu().numpy(), out.scores[:total].cpu().numpy(), sc)


def test_rnn_states_match_oracle(cuda_device):
    from dels_b200 import ops, workloads

    dev = cuda_device
    wl = workloads.cfg4(device=dev, V=2000, n_seq=9, T=16, H=320, r=64)
    t = wl.tensors
    s_scaled, s = ops.rnn_rank_states(t["x"], t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=9, T=16,
                                      want_state=True)
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    ref = O.rnn_states(f(t["x"]), f(t["w_in"]), f(t["w_s"]), f(t["bias"]), 9, 16)
    np.testing.assert_allclose(f(s), ref, rtol=2 ** -7, atol=2e-3)
    np.testing.assert_allclose(f(s_scaled), 0.3 * ref, rtol=2 ** -7, atol=2e-3)
    # RNN-fed scorer against the oracle
    out = ops.fused_argmax_bf16(t["x"], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=16, with_scores=True)
    sc = O.draft_scores(f(t["x"]), f(t["W"]), f(s_scaled), f(t["Vr"]), f(t["prior"]), np.ones(9 * 16),
                        np.full(9 * 16, 0.3))
    _check(out.tokens.cpu().numpy(), out.scores.cpu().numpy(), sc)


@pytest.mark.parametrize("n_seq,T,H,r", [(6, 7, 200, 62), (2, 5, 2048, 64)], ids=["odd_rank", "8_splits"])
def test_rnn_states_small_shapes_match_oracle(cuda_device, n_seq, T, H, r):
    """A rank that is not a multiple of 8 (W_s staged by 2-byte loads, not 16-byte rows)
    with a sequence count that leaves the last CTA partly empty; and 10 rows over a long
    K, where the input projection runs as 8 split-K partials (more than the recurrence
    loads ahead of its dot products)."""
    from dels_b200 import ops, workloads

    wl = workloads.cfg4(device=cuda_device, V=512, n_seq=n_seq, T=T, H=H, r=r)
    t = wl.tensors
    s_scaled, s = ops.rnn_rank_states(t["x"], t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=n_seq, T=T,
                                      want_state=True)
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    ref = O.rnn_states(f(t["x"]), f(t["w_in"]), f(t["w_s"]), f(t["bias"]), n_seq, T)
    np.testing.assert_allclose(f(s), ref, rtol=2 ** -7, atol=2e-3)


def _torch_scores(h, W, s_scaled, Vr, prior, beta_rows, chunk=32768):
    """fp32 reference scores on the GPU (TF32 off), chunked over the vocabulary."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        hf, sf = h.float(), s_scaled.float()
        out = torch.empty(h.shape[0], W.shape[0], dtype=torch.float32, device=h.device)
        for v0 in range(0, W.shape[0], chunk):
            v1 = min(W.shape[0], v0 + chunk)
            blk = hf @ W[v0:v1].float().T + sf @ Vr[v0:v1].float().T
            if prior is not None:
                blk -= beta_rows[:, None] * prior[None, v0:v1]
            out[:, v0:v1] = blk
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _check_full(tokens, best, ref, tol=BF16_TOL):
    """Full-size check on the GPU: tokens equal where the top-2 gap clears tol."""
    top2 = torch.topk(ref, 2, dim=1)
    ref_tok = torch.argmax(ref, dim=1)
    gap = top2.values[:, 0] - top2.values[:, 1]
    rows = torch.arange(ref.shape[0], device=ref.device)
    assert torch.all(ref[rows, tokens] >= top2.values[:, 0] - tol)
    assert torch.all((best - ref[rows, tokens]).abs() <= tol)
    clear = gap > tol
    assert torch.equal(tokens[clear], ref_tok[clear])
    return clear.float().mean().item()


def test_cfg2_full_size(cuda_device):
    """The Qwen3-8B-shape bf16 workload end to end at full size."""
    from dels_b200 import ops, workloads

    wl = workloads.cfg2(device=cuda_device)
    t = wl.tensors
    out = ops.draft_score_bf16(t["h"], t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=16,
                               with_scores=True)
    _, s_scaled = ops.rank_project_bf16(t["h"], t["w_rank"], t["alpha"], n_pos=16, want_state=False)
    pos = torch.arange(wl.rows, device=cuda_device) % 16
    ref = _torch_scores(t["h"], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"][pos])
    frac = _check_full(out.tokens, out.scores, ref)
    assert frac > 0.9
    # end-to-end against an independently computed rank state (torch, fp32 accumulate)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    s_t = (t["h"].float() @ t["w_rank"].float().T).to(torch.bfloat16).float()
    torch.backends.cuda.matmul.allow_tf32 = prev
    s_ref = (t["alpha"][pos][:, None] * s_t).to(torch.bfloat16)
    ref2 = _torch_scores(t["h"], t["W"], s_ref, t["Vr"], t["prior"], t["beta"][pos])
    _check_full(out.tokens, out.scores, ref2)


def test_cfg1_full_size_fp32(cuda_device):
    from dels_b200 import ops, workloads

    wl = workloads.cfg1(device=cuda_device)
    t = wl.tensors
    out = ops.draft_score_f32(t["h"], t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"],
                              with_scores=True)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        s = 0.3 * (t["h"].double() @ t["w_rank"].double().T)
        ref = (t["h"].double() @ t["W"].double().T + s @ t["Vr"].double().T - 0.3 * t["prior"].double()[None, :])
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    _check_full(out.tokens, out.scores.double(), ref, tol=1e-5)


def test_cfg4_full_size(cuda_device):
    from dels_b200 import ops, workloads

    wl = workloads.cfg4(device=cuda_device)
    t = wl.tensors
    s_scaled, _ = ops.rnn_rank_states(t["x"], t["w_in"], t["w_s"], t["bias"], t["alpha"], n_seq=512, T=16)
    out = ops.fused_argmax_bf16(t["x"], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"], n_pos=16,
                                with_scores=True)
    # recurrence against a float64 torch recurrence on 32 sequences
    x = t["x"][: 32 * 16].double()
    pre = (x @ t["w_in"].double().T).view(32, 16, -1)
    s = torch.zeros(32, pre.shape[-1], dtype=torch.float64, device=cuda_device)
    ref_s = []
    for step in range(16):
        s = torch.tanh(pre[:, step] + s @ t["w_s"].double().T)
        ref_s.append(s)
    ref_s = torch.stack(ref_s, 1).reshape(32 * 16, -1)
    assert torch.allclose(s_scaled[: 32 * 16].double(), 0.3 * ref_s, rtol=2 ** -7, atol=2e-3)
    rows = 1024
    ref = _torch_scores(t["x"][:rows], t["W"], s_scaled[:rows], t["Vr"], t["prior"],
                        torch.full((rows,), 0.3, device=cuda_device))
    _check_full(out.tokens[:rows], out.scores[:rows], ref)


def test_cfg3_full_size(cuda_device):
    from dels_b200 import ops, workloads

    wl = workloads.cfg3(device=cuda_device)
    t = wl.tensors
    acc, off = ops.accept_offsets(t["draft"], t["target"])
    ref_acc, ref_off = O.accept_offsets(t["draft"].cpu().numpy(), t["target"].cpu().numpy())
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(off.cpu().numpy(), ref_off)
    packed, row_pos = ops.pack_rows(t["hidden"], acc, off)
    out = ops.draft_score_bf16(packed, t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=16,
                               row_pos=row_pos, rows_dev=off[-1:], with_scores=True)
    total = int(off[-1])
    _, s_scaled = ops.rank_project_bf16(packed[:total], t["w_rank"], t["alpha"], n_pos=16, row_pos=row_pos[:total],
                                        want_state=False)
    ref = _torch_scores(packed[:total], t["W"], s_scaled, t["Vr"], t["prior"], t["beta"][row_pos[:total].long()])
    _check_full(out.tokens[:total], out.scores[:total], ref)


def test_cfg5_full_size(cuda_device):
    """The vocabulary-sharded configuration at full size on one GPU: 16384 rows over the
    whole 151936-token vocabulary against the fp32 torch reference, then the 8 contiguous
    vocabulary slices an 8-GPU run would own, each scored with global-index keys
    (keys_only), whose element-wise maximum must decode to exactly the unsharded tokens
    and scores (the NCCL all-reduce(MAX) computes that maximum across ranks)."""
    from dels_b200 import ops, workloads

    dev = cuda_device
    wl = workloads.cfg5(device=dev)
    t = wl.tensors
    V = t["W"].shape[0]
    out = ops.draft_score_bf16(t["h"], t["W"], t["w_rank"], t["Vr"], t["prior"], t["alpha"], t["beta"], n_pos=1,
                               with_scores=True)
    _, s_scaled = ops.rank_project_bf16(t["h"], t["w_rank"], t["alpha"], n_pos=1, want_state=False)
    ref = _torch_scores(t["h"], t["W"], s_scaled, t["Vr"], t["prior"], torch.full((wl.rows,), 0.3, device=dev))
    frac = _check_full(out.tokens, out.scores, ref)
    assert frac > 0.9
    del ref
    torch.cuda.empty_cache()
    keys = None
    for rank in range(8):
        v0, v1 = workloads.shard_range(V, 8, rank)
        part = ops.draft_score_bf16(t["h"], t["W"][v0:v1], t["w_rank"], t["Vr"][v0:v1], t["prior"][v0:v1],
                                    t["alpha"], t["beta"], n_pos=1, v_begin=v0, keys_only=True)
        keys = part.keys.clone() if keys is None else torch.maximum(keys, part.keys)
    tok, sc = ops.keys_decode(keys)
    assert torch.equal(keys, out.keys)
    assert torch.equal(tok, out.tokens)
    assert torch.equal(sc, out.scores)
