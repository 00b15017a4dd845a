"""The allocation-free scorer entry point, called through the C ABI.

dels_draft_score_bf16_noalloc exists for hosts that cannot give the library device
scratch (an FFI caller with no device allocator, or a serving engine whose memory pool
already owns the GPU); it keeps its scratch in an array the library reserves on each
device.  This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.  It must pass on its own in a fresh
process as well as after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2  # bf16 score tolerance used by every bf16 parity test


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(seed, dev, rows=512, H=4096, r=256, V=20011, n_pos=16):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    h = torch.randn(rows, H, generator=g, device=dev).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w_rank = (torch.randn(r, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    Vr = (torch.randn(V, r, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    k = torch.arange(1, V + 1, dtype=torch.float64, device=dev).pow(-1.1)
    prior = torch.log(k / k.sum()).to(torch.bfloat16).float()
    alpha = torch.linspace(0.5, 0.1, n_pos, device=dev)
    beta = torch.linspace(0.3, 0.0, n_pos, device=dev)
    return h, W, w_rank, Vr, prior, alpha, beta


def _noalloc(h, W, w_rank, Vr, prior, alpha, beta, tokens, scores):
    from dels_b200 import _lib

    rows, H = h.shape
    V, r = Vr.shape
    _lib.call(
        "dels_draft_score_bf16_noalloc",
        _p(h), h.stride(0), _p(W), W.stride(0), _p(w_rank), w_rank.stride(0), _p(Vr), Vr.stride(0), _p(prior),
        _p(alpha), _p(beta), alpha.numel(), None, rows, None, H, r, V, 0, _lib.DELS_ACT_IDENTITY, None, _p(tokens),
        _p(scores), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    from dels_b200 import ops

    dev = cuda_device
    for seed in (7, 8):  # two calls in a row: the shared scratch must not leak state
        h, W, w_rank, Vr, prior, alpha, beta = _inputs(seed, dev)
        tok = torch.full((h.shape[0],), -1, dtype=torch.int64, device=dev)
        sc = torch.zeros(h.shape[0], dtype=torch.float32, device=dev)
        _noalloc(h, W, w_rank, Vr, prior, alpha, beta, tok, sc)
        ref = ops.draft_score_bf16(h, W, w_rank, Vr, prior, alpha, beta, n_pos=16, with_scores=True)
        torch.cuda.synchronize()
        assert torch.all((sc - ref.scores).abs() <= TOL)
        # same kernels on the same inputs: tokens agree (up to exact ties of the score)
        same = tok == ref.tokens
        if not bool(same.all()):
            assert torch.all((sc[~same] - ref.scores[~same]).abs() <= TOL)
        assert same.float().mean().item() > 0.99


def test_noalloc_rejects_oversized_shapes(cuda_device):
    from dels_b200 import _lib

    with pytest.raises(_lib.DelsArgumentError, match="allocation-free entry point"):
        _lib.call("dels_draft_score_bf16_noalloc", None, 8192, None, 8192, None, 8192, None, 256, None, None, None,
                  16, None, 16384, None, 8192, 256, 151936, 0, 0, None, None, None, None)
