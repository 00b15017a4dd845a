"""Failure detection on the GPU without a fault: the bounded mbarrier wait gives up,
records DELS_ERR_DEVICE_TIMEOUT in the status word, propagates the abort to the other
waiting role, and the CUDA context stays usable for the next scoring call."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    from dels_b200 import _lib, ops

    dev = cuda_device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    waited = torch.zeros(2, dtype=torch.int64, device=dev)
    _lib.call("dels_selftest_bounded_wait", ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(waited.data_ptr()),
              20.0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.DELS_ERR_DEVICE_TIMEOUT
    w0, w1 = (int(x) for x in waited.tolist())
    assert 20e6 <= w0 < 1e9  # gave up after the 20 ms limit, well before the default 2 s
    assert 0 < w1 < 1e9  # the second role left on the abort flag, not on its own 2 s limit
    # the context is intact: a scoring call right after returns correct tokens
    h = torch.zeros(3, 64, dtype=torch.bfloat16, device=dev)
    h[:, 0] = 1
    W = torch.zeros(500, 64, dtype=torch.bfloat16, device=dev)
    W[123, 0] = 1
    wr = torch.zeros(64, 64, dtype=torch.bfloat16, device=dev)
    Vr = torch.zeros(500, 64, dtype=torch.bfloat16, device=dev)
    a = torch.ones(1, device=dev)
    assert ops.draft_score_bf16(h, W, wr, Vr, None, a, a).tokens.tolist() == [123, 123, 123]
