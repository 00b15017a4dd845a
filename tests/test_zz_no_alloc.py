"""The allocation-free scorer entry point, called through the C ABI.

dels_draft_score_bf16_noalloc exists for hosts that cannot give the library device
scratch: a service that binds the C ABI through an FFI layer with no device allocator
of its own, or a serving engine whose memory pool already owns nearly all of the GPU.
It keeps its scratch in an array the library reserves on each device, and its device
status word there is read and cleared with dels_noalloc_status.

This file is collected last on purpose: if it fails, a run that stops at the first
failure has already run every other test.  It must pass on its own in a fresh process
as well as after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import dels_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2  # bf16 score tolerance used by every bf16 parity test


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(seed, dev, rows, H, r, V, n_pos=16):
    """bf16-exact host arrays (for the oracle) and their device copies."""
    rng = np.random.default_rng(seed)
    h = O.bf16_round(rng.standard_normal((rows, H)).astype(np.float32))
    W = O.bf16_round((rng.standard_normal((V, H)) * 0.02).astype(np.float32))
    w_rank = O.bf16_round((rng.standard_normal((r, H)) * 0.02).astype(np.float32))
    Vr = O.bf16_round((rng.standard_normal((V, r)) * 0.02).astype(np.float32))
    prior = O.bf16_round(O.zipf_log_prior(V).astype(np.float32))
    alpha = np.linspace(0.5, 0.1, n_pos)
    beta = np.linspace(0.3, 0.0, n_pos)
    host = (h, W, w_rank, Vr, prior, alpha, beta)

    def bf(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)

    def f32(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)

    devt = (bf(h), bf(W), bf(w_rank), bf(Vr), f32(prior), f32(alpha), f32(beta))
    return host, devt


def _noalloc(h, W, w_rank, Vr, prior, alpha, beta, tokens, scores):
    from dels_b200 import _lib

    rows, H = h.shape
    V, r = Vr.shape
    _lib.call(
        "dels_draft_score_bf16_noalloc",
        _p(h), h.stride(0), _p(W), W.stride(0), _p(w_rank), w_rank.stride(0), _p(Vr), Vr.stride(0), _p(prior),
        _p(alpha), _p(beta), alpha.numel(), None, rows, None, H, r, V, 0, _lib.DELS_ACT_IDENTITY, None, _p(tokens),
        _p(scores), _stream(),
    )


def _status(clear: bool, dev) -> int:
    from dels_b200 import _lib

    out = torch.full((1,), 12345, dtype=torch.int32, device=dev)
    _lib.call("dels_noalloc_status", _p(out), 1 if clear else 0, _stream())
    torch.cuda.synchronize()
    return int(out.item())


def _run_noalloc(devt, dev):
    h = devt[0]
    tok = torch.full((h.shape[0],), -1, dtype=torch.int64, device=dev)
    sc = torch.full((h.shape[0],), float("nan"), dtype=torch.float32, device=dev)
    _noalloc(*devt, tok, sc)
    return tok, sc


def test_noalloc_matches_oracle(cuda_device):
    """Against the float64 oracle, at sizes it finishes in seconds: the single-CTA tile
    scorer (100 rows) and the CTA-pair scorer (300 rows)."""
    dev = cuda_device
    for seed, rows in ((11, 100), (12, 300)):
        host, devt = _inputs(seed, dev, rows=rows, H=512, r=64, V=5003)
        tok, sc = _run_noalloc(devt, dev)
        torch.cuda.synchronize()
        h, W, w_rank, Vr, prior, alpha, beta = host
        _, ref_scores, _ = O.draft_score_bf16(h, W, w_rank, Vr, prior, alpha, beta, n_pos=16)
        tok, sc = tok.cpu().numpy(), sc.cpu().numpy()
        ref_tok = O.argmax_first(ref_scores)
        gap = O.top2_gap(ref_scores)
        idx = np.arange(rows)
        np.testing.assert_allclose(sc, ref_scores[idx, tok], rtol=0, atol=TOL)
        assert np.all(ref_scores[idx, tok] >= ref_scores[idx, ref_tok] - TOL)
        clear = gap > TOL
        assert clear.mean() > 0.5
        np.testing.assert_array_equal(tok[clear], ref_tok[clear])
    assert _status(clear=False, dev=dev) == 0


def test_noalloc_equals_workspace_entry_point_twice(cuda_device):
    """The same kernels as dels_draft_score_bf16 on the same inputs, with a deterministic
    split-K and an exact key maximum: tokens and scores are bit-identical.  Two calls in a
    row, the second with fewer rows than the first, so a key, partial sum or counter left
    in the shared array by the first call would show up in the second."""
    from dels_b200 import ops

    dev = cuda_device
    for seed, rows in ((7, 512), (8, 40)):
        _, devt = _inputs(seed, dev, rows=rows, H=4096, r=256, V=20011)
        tok, sc = _run_noalloc(devt, dev)
        ref = ops.draft_score_bf16(*devt, n_pos=16, with_scores=True)
        torch.cuda.synchronize()
        assert torch.equal(tok, ref.tokens)
        assert torch.equal(sc, ref.scores)
    assert _status(clear=False, dev=dev) == 0


def test_noalloc_status_reports_and_clears_a_device_timeout(cuda_device):
    """A bounded wait that gives up records DELS_ERR_DEVICE_TIMEOUT in the allocation-free
    status word (no fault: the wait returns after 20 ms); dels_noalloc_status reads it,
    it stays set until cleared, and scoring calls after the clear leave it at zero."""
    from dels_b200 import _lib

    dev = cuda_device
    assert _status(clear=True, dev=dev) == 0
    waited = torch.zeros(2, dtype=torch.int64, device=dev)
    _lib.call("dels_selftest_bounded_wait_noalloc", _p(waited), 20.0, _stream())
    torch.cuda.synchronize()
    assert int(waited[0].item()) >= 20e6
    assert _status(clear=False, dev=dev) == _lib.DELS_ERR_DEVICE_TIMEOUT  # sticky
    assert _status(clear=True, dev=dev) == _lib.DELS_ERR_DEVICE_TIMEOUT  # read, then cleared
    assert _status(clear=False, dev=dev) == 0
    host, devt = _inputs(13, dev, rows=16, H=256, r=64, V=4099)
    tok, _ = _run_noalloc(devt, dev)
    torch.cuda.synchronize()
    h, W, w_rank, Vr, prior, alpha, beta = host
    _, ref_scores, _ = O.draft_score_bf16(h, W, w_rank, Vr, prior, alpha, beta, n_pos=16)
    clear = O.top2_gap(ref_scores) > TOL
    np.testing.assert_array_equal(tok.cpu().numpy()[clear], O.argmax_first(ref_scores)[clear])
    assert _status(clear=False, dev=dev) == 0


def test_noalloc_rejects_oversized_shapes(cuda_device):
    from dels_b200 import _lib

    with pytest.raises(_lib.DelsArgumentError, match="allocation-free entry point"):
        _lib.call("dels_draft_score_bf16_noalloc", None, 8192, None, 8192, None, 8192, None, 256, None, None, None,
                  16, None, 16384, None, 8192, 256, 151936, 0, 0, None, None, None, None)
