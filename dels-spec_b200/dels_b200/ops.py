"""Torch-facing wrappers of the C ABI (``include/dels_b200.h``).

Every function takes CUDA tensors, checks dtypes and shapes, and enqueues the CUDA
kernels on the current stream through :mod:`dels_b200._lib`.  Outputs can be passed in
(``out=`` arguments) so that callers which capture CUDA graphs allocate nothing per
call.  There is deliberately no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

ACTIVATIONS = {"identity": _lib.DELS_ACT_IDENTITY, "silu": _lib.DELS_ACT_SILU}


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(name: str, t: torch.Tensor, dtype: torch.dtype, ndim: int | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); there is no CPU path")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype} (got {t.dtype})")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D (got shape {tuple(t.shape)})")


def _row_major(name: str, t: torch.Tensor) -> int:
    """Leading dimension (elements) of a 2-D tensor with unit column stride."""
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D (got shape {tuple(t.shape)})")
    if t.numel() == 0:
        return max(int(t.shape[1]), 1)
    if t.stride(1) != 1 and t.shape[1] > 1:
        raise ValueError(f"{name} must have contiguous rows (stride {tuple(t.stride())})")
    return t.stride(0) if t.shape[0] > 1 else max(t.stride(0), int(t.shape[1]))


def _f32_vec(name: str, t: torch.Tensor | None, device: torch.device) -> torch.Tensor | None:
    if t is None:
        return None
    _require_cuda(name, t, torch.float32, 1)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t


def _i32_vec(name: str, t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    _require_cuda(name, t, torch.int32, 1)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def init(device: torch.device | int | None = None) -> None:
    """Load the kernels on ``device`` (do this before capturing a CUDA graph)."""
    if device is None:
        index = torch.cuda.current_device()
    elif isinstance(device, int):
        index = device
    else:
        index = torch.device(device).index
        index = torch.cuda.current_device() if index is None else index
    _lib.call("dels_init", int(index))


class Workspace:
    """Zero-initialised, 256-byte-aligned device scratch owned by the caller.

    The first 8 bytes hold the completion counter and the device status word that the
    kernels use; :meth:`status` reads the latter (one device-to-host copy)."""

    def __init__(self, nbytes: int, device: torch.device):
        nbytes = max(int(nbytes), _lib.DELS_WS_HEADER_BYTES)
        self._raw = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        off = (-self._raw.data_ptr()) % 256
        self.buf = self._raw[off : off + nbytes]
        self.nbytes = nbytes
        self.device = device

    def ensure(self, nbytes: int) -> "Workspace":
        return self if nbytes <= self.nbytes else Workspace(nbytes, self.device)

    @property
    def ptr(self) -> ctypes.c_void_p:
        return ctypes.c_void_p(self.buf.data_ptr())

    def status(self) -> int:
        return int(self.buf[4:8].view(torch.int32).item())

    def clear_status(self) -> None:
        self.buf[4:8].zero_()

    def check(self) -> None:
        """Raise if a kernel recorded a device-side failure (synchronises)."""
        st = self.status()
        if st != 0:
            self.clear_status()
            raise _lib.DelsError("device", st, _lib.load().dels_status_string(st).decode())


_ws_cache: dict[tuple[int, int], Workspace] = {}


def workspace(nbytes: int, device: torch.device) -> Workspace:
    """A cached workspace per (device, stream) large enough for ``nbytes``."""
    key = (device.index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.nbytes < nbytes:
        ws = Workspace(max(nbytes, 1 << 20), device)
        _ws_cache[key] = ws
    return ws


def _positions(n_pos: int | None, alpha: torch.Tensor | None, beta: torch.Tensor | None) -> int:
    if n_pos is not None:
        return int(n_pos)
    for t in (alpha, beta):
        if t is not None:
            return int(t.numel())
    return 1


# --------------------------------------------------------------------------- scorer
@dataclass
class ScoreOut:
    tokens: torch.Tensor  # int64 [rows]
    scores: torch.Tensor | None  # fp32 [rows]
    keys: torch.Tensor  # int64 [rows] packed (score, index) keys


def draft_score_bf16(
    h: torch.Tensor,
    W: torch.Tensor,
    w_rank: torch.Tensor,
    Vr: torch.Tensor,
    prior: torch.Tensor | None,
    alpha: torch.Tensor,
    beta: torch.Tensor,
    *,
    n_pos: int | None = None,
    row_pos: torch.Tensor | None = None,
    rows_dev: torch.Tensor | None = None,
    v_begin: int = 0,
    activation: str = "identity",
    keys_only: bool = False,
    with_scores: bool = False,
    out: ScoreOut | None = None,
    ws: Workspace | None = None,
) -> ScoreOut:
    """argmax_v (h.W[v] + alpha_p * act(h.w_rank^T).Vr[v] - beta_p * prior[v]) per row.

    ``W``/``Vr``/``prior`` may be one rank's contiguous vocabulary slice starting at
    global index ``v_begin``; with ``keys_only=True`` the packed keys are returned
    undecoded for a cross-rank all-reduce(MAX) (then :func:`keys_decode`)."""
    dev = h.device
    for name, t in (("h", h), ("W", W), ("w_rank", w_rank), ("Vr", Vr)):
        _require_cuda(name, t, torch.bfloat16, 2)
    rows, H = h.shape
    V = W.shape[0]
    r = w_rank.shape[0]
    if W.shape[1] != H or w_rank.shape[1] != H or Vr.shape != (V, r):
        raise ValueError(f"shape mismatch: h {tuple(h.shape)}, W {tuple(W.shape)}, w_rank {tuple(w_rank.shape)}, "
                         f"Vr {tuple(Vr.shape)}")
    prior = _f32_vec("prior", prior, dev)
    alpha = _f32_vec("alpha", alpha, dev)
    beta = _f32_vec("beta", beta, dev)
    row_pos = _i32_vec("row_pos", row_pos)
    rows_dev = _i32_vec("rows_dev", rows_dev)
    if prior is not None and prior.numel() != V:
        raise ValueError(f"prior has {prior.numel()} entries, expected {V}")
    npos = _positions(n_pos, alpha, beta)
    if out is None:
        out = ScoreOut(
            tokens=torch.empty(rows, dtype=torch.int64, device=dev),
            scores=torch.empty(rows, dtype=torch.float32, device=dev) if with_scores else None,
            keys=torch.empty(rows, dtype=torch.int64, device=dev),
        )
    need = _lib.query("dels_score_workspace_bytes", rows, H, r)
    ws = workspace(need, dev) if ws is None else ws.ensure(need)
    _lib.call(
        "dels_draft_score_bf16",
        _ptr(h), _row_major("h", h),
        _ptr(W), _row_major("W", W), _ptr(w_rank), _row_major("w_rank", w_rank), _ptr(Vr), _row_major("Vr", Vr),
        _ptr(prior), _ptr(alpha), _ptr(beta), npos, _ptr(row_pos), rows, _ptr(rows_dev), H, r, V, int(v_begin),
        ACTIVATIONS[activation], _ptr(out.keys), None if keys_only else _ptr(out.tokens),
        None if (keys_only or out.scores is None) else _ptr(out.scores), ws.ptr, ws.nbytes, _stream(dev),
    )
    return out


def rank_project_bf16(
    x: torch.Tensor,
    w_rank: torch.Tensor,
    alpha: torch.Tensor | None,
    *,
    n_pos: int | None = None,
    row_pos: torch.Tensor | None = None,
    activation: str = "identity",
    s_out: torch.Tensor | None = None,
    s_scaled: torch.Tensor | None = None,
    keys: torch.Tensor | None = None,
    want_state: bool = True,
    ws: Workspace | None = None,
) -> tuple[torch.Tensor | None, torch.Tensor]:
    """(s, alpha_p * s) with s = bf16(act(bf16(x . w_rank^T))); optionally resets keys."""
    dev = x.device
    _require_cuda("x", x, torch.bfloat16, 2)
    _require_cuda("w_rank", w_rank, torch.bfloat16, 2)
    rows, K = x.shape
    r = w_rank.shape[0]
    if w_rank.shape[1] != K:
        raise ValueError(f"w_rank {tuple(w_rank.shape)} does not match x {tuple(x.shape)}")
    alpha = _f32_vec("alpha", alpha, dev)
    row_pos = _i32_vec("row_pos", row_pos)
    if s_scaled is None:
        s_scaled = torch.empty(rows, r, dtype=torch.bfloat16, device=dev)
    if want_state and s_out is None:
        s_out = torch.empty(rows, r, dtype=torch.bfloat16, device=dev)
    need = _lib.query("dels_rank_workspace_bytes", rows, K, r)
    ws = workspace(need, dev) if ws is None else ws.ensure(need)
    _lib.call(
        "dels_rank_project_bf16",
        _ptr(x), _row_major("x", x), _ptr(w_rank), _row_major("w_rank", w_rank), rows, K, r, ACTIVATIONS[activation],
        _ptr(alpha), _positions(n_pos, alpha, None), _ptr(row_pos), _ptr(s_out), _ptr(s_scaled), _ptr(keys),
        ws.ptr, ws.nbytes, _stream(dev),
    )
    return s_out, s_scaled


def fused_argmax_bf16(
    h: torch.Tensor,
    W: torch.Tensor,
    s_scaled: torch.Tensor,
    Vr: torch.Tensor,
    prior: torch.Tensor | None,
    beta: torch.Tensor,
    *,
    n_pos: int | None = None,
    row_pos: torch.Tensor | None = None,
    rows_dev: torch.Tensor | None = None,
    v_begin: int = 0,
    keys_ready: bool = False,
    keys_only: bool = False,
    with_scores: bool = False,
    out: ScoreOut | None = None,
    ws: Workspace | None = None,
) -> ScoreOut:
    """Scorer with a precomputed bf16 operand ``s_scaled`` = alpha_p * rank state."""
    dev = h.device
    for name, t in (("h", h), ("W", W), ("s_scaled", s_scaled), ("Vr", Vr)):
        _require_cuda(name, t, torch.bfloat16, 2)
    rows, H = h.shape
    V, r = Vr.shape
    if W.shape != (V, H) or s_scaled.shape != (rows, r):
        raise ValueError("shape mismatch between h, W, s_scaled and Vr")
    prior = _f32_vec("prior", prior, dev)
    beta = _f32_vec("beta", beta, dev)
    if out is None:
        out = ScoreOut(
            tokens=torch.empty(rows, dtype=torch.int64, device=dev),
            scores=torch.empty(rows, dtype=torch.float32, device=dev) if with_scores else None,
            keys=torch.empty(rows, dtype=torch.int64, device=dev),
        )
    ws = workspace(_lib.DELS_WS_HEADER_BYTES, dev) if ws is None else ws
    _lib.call(
        "dels_fused_argmax_bf16",
        _ptr(h), _row_major("h", h), _ptr(W), _row_major("W", W), _ptr(s_scaled), _row_major("s_scaled", s_scaled),
        _ptr(Vr), _row_major("Vr", Vr), _ptr(prior), _ptr(beta), _positions(n_pos, None, beta),
        _ptr(_i32_vec("row_pos", row_pos)), rows, _ptr(_i32_vec("rows_dev", rows_dev)), H, r, V, int(v_begin),
        _lib.DELS_FLAG_KEYS_READY if keys_ready else 0, _ptr(out.keys), None if keys_only else _ptr(out.tokens),
        None if (keys_only or out.scores is None) else _ptr(out.scores), ws.ptr, ws.nbytes, _stream(dev),
    )
    return out


def fused_argmax_base_bf16(
    base: torch.Tensor,
    s_scaled: torch.Tensor,
    Vr: torch.Tensor,
    prior: torch.Tensor | None,
    beta: torch.Tensor,
    *,
    n_pos: int | None = None,
    row_pos: torch.Tensor | None = None,
    v_begin: int = 0,
    keys_ready: bool = False,
    with_scores: bool = False,
    out: ScoreOut | None = None,
    ws: Workspace | None = None,
) -> ScoreOut:
    """Runner step: argmax_v(base[i, v] + s_scaled[i].Vr[v] - beta_p prior[v])."""
    dev = base.device
    for name, t in (("base", base), ("s_scaled", s_scaled), ("Vr", Vr)):
        _require_cuda(name, t, torch.bfloat16, 2)
    rows, V = base.shape
    r = Vr.shape[1]
    if Vr.shape[0] != V or s_scaled.shape != (rows, r):
        raise ValueError("shape mismatch between base, s_scaled and Vr")
    prior = _f32_vec("prior", prior, dev)
    beta = _f32_vec("beta", beta, dev)
    if out is None:
        out = ScoreOut(
            tokens=torch.empty(rows, dtype=torch.int64, device=dev),
            scores=torch.empty(rows, dtype=torch.float32, device=dev) if with_scores else None,
            keys=torch.empty(rows, dtype=torch.int64, device=dev),
        )
    ws = workspace(_lib.DELS_WS_HEADER_BYTES, dev) if ws is None else ws
    _lib.call(
        "dels_fused_argmax_base_bf16",
        _ptr(base), _row_major("base", base), _ptr(s_scaled), _row_major("s_scaled", s_scaled), _ptr(Vr),
        _row_major("Vr", Vr), _ptr(prior), _ptr(beta), _positions(n_pos, None, beta),
        _ptr(_i32_vec("row_pos", row_pos)), rows, None, r, V, int(v_begin),
        _lib.DELS_FLAG_KEYS_READY if keys_ready else 0, _ptr(out.keys), _ptr(out.tokens),
        None if out.scores is None else _ptr(out.scores), ws.ptr, ws.nbytes, _stream(dev),
    )
    return out


def fused_argmax_base_gru_bf16(
    base: torch.Tensor,
    s_scaled: torch.Tensor,
    Vr: torch.Tensor,
    prior: torch.Tensor | None,
    beta: torch.Tensor,
    w_hh: torch.Tensor,
    b_hh: torch.Tensor | None,
    h: torch.Tensor,
    gh_out: torch.Tensor,
    *,
    keys_ready: bool = False,
    out: ScoreOut,
    ws: Workspace,
) -> ScoreOut:
    """fused_argmax_base_bf16 for a rollout step of at most 4 rows that also computes the
    next step's gh_out = bf16(w_hh . h + b_hh) in the same launch."""
    dev = base.device
    for name, t in (("base", base), ("s_scaled", s_scaled), ("Vr", Vr), ("w_hh", w_hh), ("h", h), ("gh_out", gh_out)):
        _require_cuda(name, t, torch.bfloat16, 2)
    rows, V = base.shape
    r = Vr.shape[1]
    G = h.shape[1]
    if Vr.shape[0] != V or s_scaled.shape != (rows, r):
        raise ValueError("shape mismatch between base, s_scaled and Vr")
    if w_hh.shape != (3 * G, G) or not w_hh.is_contiguous() or h.shape != (rows, G) or not h.is_contiguous() \
            or gh_out.shape != (rows, 3 * G) or not gh_out.is_contiguous():
        raise ValueError("GRU operands do not match")
    _lib.call(
        "dels_fused_argmax_base_gru_bf16",
        _ptr(base), _row_major("base", base), _ptr(s_scaled), _row_major("s_scaled", s_scaled), _ptr(Vr),
        _row_major("Vr", Vr), _ptr(_f32_vec("prior", prior, dev)), _ptr(_f32_vec("beta", beta, dev)),
        _positions(None, None, beta), rows, r, V, _lib.DELS_FLAG_KEYS_READY if keys_ready else 0, _ptr(out.keys),
        _ptr(out.tokens), ws.ptr, ws.nbytes, _ptr(w_hh), _ptr(b_hh), _ptr(h), G, _ptr(gh_out), _stream(dev),
    )
    return out


def draft_score_f32(
    h: torch.Tensor,
    W: torch.Tensor,
    w_rank: torch.Tensor,
    Vr: torch.Tensor,
    prior: torch.Tensor | None,
    alpha: torch.Tensor,
    beta: torch.Tensor,
    *,
    n_pos: int | None = None,
    row_pos: torch.Tensor | None = None,
    v_begin: int = 0,
    keys_only: bool = False,
    with_scores: bool = False,
    out: ScoreOut | None = None,
    ws: Workspace | None = None,
) -> ScoreOut:
    """fp32 scorer (CUDA cores): argmax_v(h.W[v] + (alpha_p h.w_rank^T).Vr[v] - beta_p prior[v])."""
    dev = h.device
    for name, t in (("h", h), ("W", W), ("w_rank", w_rank), ("Vr", Vr)):
        _require_cuda(name, t, torch.float32, 2)
    rows, H = h.shape
    V = W.shape[0]
    r = w_rank.shape[0]
    if W.shape[1] != H or w_rank.shape[1] != H or Vr.shape != (V, r):
        raise ValueError("shape mismatch between h, W, w_rank and Vr")
    prior = _f32_vec("prior", prior, dev)
    alpha = _f32_vec("alpha", alpha, dev)
    beta = _f32_vec("beta", beta, dev)
    if out is None:
        out = ScoreOut(
            tokens=torch.empty(rows, dtype=torch.int64, device=dev),
            scores=torch.empty(rows, dtype=torch.float32, device=dev) if with_scores else None,
            keys=torch.empty(rows, dtype=torch.int64, device=dev),
        )
    need = _lib.query("dels_score_f32_workspace_bytes", rows, H, r)
    ws = workspace(need, dev) if ws is None else ws.ensure(need)
    _lib.call(
        "dels_draft_score_f32",
        _ptr(h), _row_major("h", h), _ptr(W), _row_major("W", W), _ptr(w_rank), _row_major("w_rank", w_rank),
        _ptr(Vr), _row_major("Vr", Vr), _ptr(prior), _ptr(alpha), _ptr(beta), _positions(n_pos, alpha, beta),
        _ptr(_i32_vec("row_pos", row_pos)), rows, H, r, V, int(v_begin), _ptr(out.keys),
        None if keys_only else _ptr(out.tokens), None if (keys_only or out.scores is None) else _ptr(out.scores),
        ws.ptr, ws.nbytes, _stream(dev),
    )
    return out


def keys_init(keys: torch.Tensor, ws: Workspace | None = None) -> None:
    _require_cuda("keys", keys, torch.int64, 1)
    _lib.call("dels_keys_init", _ptr(keys), keys.numel(), None if ws is None else ws.ptr, _stream(keys.device))


def keys_decode(
    keys: torch.Tensor,
    *,
    rows_dev: torch.Tensor | None = None,
    tokens: torch.Tensor | None = None,
    scores: torch.Tensor | None = None,
    with_scores: bool = True,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Token ids (int64) and scores (fp32) from packed keys."""
    _require_cuda("keys", keys, torch.int64, 1)
    n = keys.numel()
    if tokens is None:
        tokens = torch.empty(n, dtype=torch.int64, device=keys.device)
    if with_scores and scores is None:
        scores = torch.empty(n, dtype=torch.float32, device=keys.device)
    _lib.call("dels_keys_decode", _ptr(keys), n, _ptr(_i32_vec("rows_dev", rows_dev)), _ptr(tokens), _ptr(scores),
              _stream(keys.device))
    return tokens, scores


# --------------------------------------------------------------------------- acceptance
def accept_offsets(
    draft: torch.Tensor,
    target: torch.Tensor,
    *,
    commit_extra: int = 0,
    accept: torch.Tensor | None = None,
    offsets: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-sequence accepted prefix lengths (int32) and packed row offsets (int32, n+1)."""
    _require_cuda("draft", draft, torch.int64, 2)
    _require_cuda("target", target, torch.int64, 2)
    n_seq, n_draft = draft.shape
    if target.shape[0] != n_seq or target.shape[1] < n_draft:
        raise ValueError(f"target {tuple(target.shape)} must be [n_seq, >= {n_draft}]")
    dev = draft.device
    if accept is None:
        accept = torch.empty(n_seq, dtype=torch.int32, device=dev)
    if offsets is None:
        offsets = torch.empty(n_seq + 1, dtype=torch.int32, device=dev)
    _lib.call("dels_accept_offsets", _ptr(draft), _row_major("draft", draft), _ptr(target),
              _row_major("target", target), n_seq, n_draft, int(commit_extra), _ptr(accept), _ptr(offsets),
              _stream(dev))
    return accept, offsets


def pack_rows(
    hidden: torch.Tensor,
    accept: torch.Tensor,
    offsets: torch.Tensor,
    *,
    packed: torch.Tensor | None = None,
    row_pos: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather hidden[b, j] for j < accept[b] into rows offsets[b] + j (capacity n_seq*P)."""
    _require_cuda("hidden", hidden, torch.bfloat16, 3)
    n_seq, P, H = hidden.shape
    if hidden.stride(2) != 1:
        raise ValueError("hidden must have contiguous rows")
    dev = hidden.device
    if packed is None:
        packed = torch.empty(n_seq * P, H, dtype=torch.bfloat16, device=dev)
    if row_pos is None:
        row_pos = torch.zeros(n_seq * P, dtype=torch.int32, device=dev)
    _lib.call("dels_pack_rows_bf16", _ptr(hidden), hidden.stride(0), hidden.stride(1), n_seq, P, H,
              _ptr(_i32_vec("accept", accept)), _ptr(_i32_vec("offsets", offsets)), _ptr(packed),
              _row_major("packed", packed), _ptr(row_pos), _stream(dev))
    return packed, row_pos


# --------------------------------------------------------------------------- RNN head
def rnn_rank_states(
    x: torch.Tensor,
    w_in: torch.Tensor,
    w_s: torch.Tensor,
    bias: torch.Tensor | None,
    alpha: torch.Tensor,
    *,
    n_seq: int,
    T: int,
    s_scaled: torch.Tensor | None = None,
    s_out: torch.Tensor | None = None,
    want_state: bool = False,
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """alpha_t * s_t (bf16) for s_t = tanh(W_in x_t + W_s s_{t-1} + b), s_0 = 0."""
    dev = x.device
    _require_cuda("x", x, torch.bfloat16, 2)
    _require_cuda("w_in", w_in, torch.bfloat16, 2)
    _require_cuda("w_s", w_s, torch.bfloat16, 2)
    rows, H = x.shape
    r = w_in.shape[0]
    if rows != n_seq * T or w_in.shape[1] != H or w_s.shape != (r, r) or not w_s.is_contiguous():
        raise ValueError("shape mismatch between x, w_in and w_s")
    bias = _f32_vec("bias", bias, dev)
    alpha = _f32_vec("alpha", alpha, dev)
    if s_scaled is None:
        s_scaled = torch.empty(rows, r, dtype=torch.bfloat16, device=dev)
    if want_state and s_out is None:
        s_out = torch.empty(rows, r, dtype=torch.bfloat16, device=dev)
    need = _lib.query("dels_rnn_workspace_bytes", n_seq, T, H, r)
    ws = workspace(need, dev) if ws is None else ws.ensure(need)
    _lib.call("dels_rnn_rank_states_bf16", _ptr(x), _row_major("x", x), _ptr(w_in), _row_major("w_in", w_in),
              _ptr(w_s), _ptr(bias), _ptr(alpha), n_seq, T, H, r, _ptr(s_scaled), _ptr(s_out), _ptr(keys), ws.ptr,
              ws.nbytes, _stream(dev))
    return s_scaled, s_out


# --------------------------------------------------------------------------- rollout kernels
def gru_step(
    tokens: torch.Tensor,
    gi_table: torch.Tensor,
    w_hh: torch.Tensor,
    h_in: torch.Tensor | None,
    h_out: torch.Tensor,
    *,
    b_hh: torch.Tensor | None = None,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """h_out = GRU(gi_table[tokens], h_in) with gh = W_hh h_in (+ b_hh); h_in None = zeros.
    With ``tokens_are_keys`` the tokens are the previous step's packed (score, index) keys."""
    _require_cuda("tokens", tokens, torch.int64)
    _require_cuda("gi_table", gi_table, torch.bfloat16, 2)
    _require_cuda("w_hh", w_hh, torch.bfloat16, 2)
    _require_cuda("h_out", h_out, torch.bfloat16, 2)
    B, G = h_out.shape
    V = gi_table.shape[0]
    if w_hh.shape != (3 * G, G) or not w_hh.is_contiguous() or gi_table.shape[1] != 3 * G:
        raise ValueError("GRU weights do not match the hidden size")
    if h_in is not None and (h_in.shape != (B, G) or not h_in.is_contiguous()):
        raise ValueError("h_in must be a contiguous [B, G] tensor")
    if not h_out.is_contiguous():
        raise ValueError("h_out must be contiguous")
    tok_stride = tokens.stride(0) if tokens.dim() >= 1 and tokens.numel() > 1 else 1
    _lib.call("dels_gru_step_bf16", _ptr(tokens), tok_stride, int(bool(tokens_are_keys)), _ptr(gi_table),
              _row_major("gi_table", gi_table),
              _ptr(w_hh), _ptr(b_hh), _ptr(h_in), _ptr(h_out), B, G, V, None if ws is None else ws.ptr,
              _stream(h_out.device))
    return h_out


def gru_gates(
    tokens: torch.Tensor,
    gi_table: torch.Tensor,
    gh: torch.Tensor,
    h_in: torch.Tensor | None,
    h_out: torch.Tensor,
    *,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """h_out = GRU gates(gi_table[tokens], gh, h_in) for a precomputed gh = bf16(W_hh h + b_hh).
    With ``tokens_are_keys`` the tokens are the previous step's packed (score, index) keys."""
    _require_cuda("tokens", tokens, torch.int64)
    _require_cuda("gi_table", gi_table, torch.bfloat16, 2)
    _require_cuda("gh", gh, torch.bfloat16, 2)
    _require_cuda("h_out", h_out, torch.bfloat16, 2)
    B, G = h_out.shape
    V = gi_table.shape[0]
    if gh.shape != (B, 3 * G) or gh.stride(1) != 1 or gi_table.shape[1] != 3 * G or not h_out.is_contiguous():
        raise ValueError("GRU gate operands do not match the hidden size")
    if h_in is not None and (h_in.shape != (B, G) or not h_in.is_contiguous()):
        raise ValueError("h_in must be a contiguous [B, G] tensor")
    tok_stride = tokens.stride(0) if tokens.dim() >= 1 and tokens.numel() > 1 else 1
    _lib.call("dels_gru_gates_bf16", _ptr(tokens), tok_stride, int(bool(tokens_are_keys)), _ptr(gi_table),
              _row_major("gi_table", gi_table),
              _ptr(gh), gh.stride(0), _ptr(h_in), _ptr(h_out), B, G, V, None if ws is None else ws.ptr,
              _stream(h_out.device))
    return h_out


def gru_step_tc(
    tokens: torch.Tensor,
    gi_table: torch.Tensor,
    w_hh: torch.Tensor,
    h_in: torch.Tensor,
    h_out: torch.Tensor,
    *,
    b_hh: torch.Tensor | None = None,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """h_out = GRU(gi_table[tokens], h_in) with gh = bf16(W_hh h_in + b_hh) from a tensor-core
    split-K GEMM whose finalisation evaluates the gates (bit-identical to linear_bf16 followed
    by gru_gates).  With ``tokens_are_keys`` the tokens are packed (score, index) keys."""
    _require_cuda("tokens", tokens, torch.int64)
    _require_cuda("gi_table", gi_table, torch.bfloat16, 2)
    _require_cuda("w_hh", w_hh, torch.bfloat16, 2)
    _require_cuda("h_in", h_in, torch.bfloat16, 2)
    _require_cuda("h_out", h_out, torch.bfloat16, 2)
    B, G = h_out.shape
    V = gi_table.shape[0]
    if w_hh.shape != (3 * G, G) or not w_hh.is_contiguous() or gi_table.shape[1] != 3 * G:
        raise ValueError("GRU weights do not match the hidden size")
    if h_in.shape != (B, G) or not h_in.is_contiguous() or not h_out.is_contiguous():
        raise ValueError("h_in / h_out must be contiguous [B, G] tensors")
    need = _lib.query("dels_gru_step_tc_workspace_bytes", B, G)
    ws = workspace(need, h_out.device) if ws is None else ws.ensure(need)
    tok_stride = tokens.stride(0) if tokens.dim() >= 1 and tokens.numel() > 1 else 1
    _lib.call("dels_gru_step_tc_bf16", _ptr(tokens), tok_stride, int(bool(tokens_are_keys)), _ptr(gi_table),
              _row_major("gi_table", gi_table),
              _ptr(w_hh), _ptr(b_hh), _ptr(h_in), _ptr(h_out), B, G, V, ws.ptr, ws.nbytes, _stream(h_out.device))
    return h_out


def gru_rank_gemv(
    tokens: torch.Tensor,
    gi_table: torch.Tensor,
    gh: torch.Tensor,
    h_in: torch.Tensor | None,
    h_out: torch.Tensor,
    w_rank: torch.Tensor,
    alpha: torch.Tensor | None,
    s_scaled: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    activation: str = "identity",
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """One small-batch rollout step: h_out = GRU gates(gi_table[tokens], gh, h_in) (gh =
    bf16(W_hh h_in + b_hh) from an earlier rank_gemv), then s_scaled = bf16(alpha[0] *
    act(w_rank . h_out + bias)) in the same launch.  ``tokens_are_keys``: ``tokens`` holds
    the previous step's packed argmax keys (a keys-only scorer call), decoded here."""
    _require_cuda("tokens", tokens, torch.int64)
    _require_cuda("gi_table", gi_table, torch.bfloat16, 2)
    _require_cuda("gh", gh, torch.bfloat16, 2)
    _require_cuda("h_out", h_out, torch.bfloat16, 2)
    _require_cuda("w_rank", w_rank, torch.bfloat16, 2)
    B, G = h_out.shape
    V = gi_table.shape[0]
    r = w_rank.shape[0]
    if gh.shape != (B, 3 * G) or gh.stride(1) != 1 or gi_table.shape[1] != 3 * G or not h_out.is_contiguous():
        raise ValueError("GRU gate operands do not match the hidden size")
    if h_in is not None and (h_in.shape != (B, G) or not h_in.is_contiguous()):
        raise ValueError("h_in must be a contiguous [B, G] tensor")
    if w_rank.shape[1] != G or s_scaled.shape != (B, r) or not s_scaled.is_contiguous():
        raise ValueError("rank projection shapes do not match")
    tok_stride = tokens.stride(0) if tokens.dim() >= 1 and tokens.numel() > 1 else 1
    _lib.call("dels_gru_rank_gemv_bf16", _ptr(tokens), tok_stride, int(tokens_are_keys), _ptr(gi_table),
              _row_major("gi_table", gi_table),
              _ptr(gh), gh.stride(0), _ptr(h_in), _ptr(h_out), B, G, V, _ptr(w_rank), _row_major("w_rank", w_rank),
              _ptr(bias), r, ACTIVATIONS[activation], _ptr(alpha), _ptr(s_scaled), _ptr(keys),
              None if ws is None else ws.ptr, _stream(h_out.device))
    return s_scaled


def gru_correction_mid(
    tokens: torch.Tensor,
    gi_table: torch.Tensor,
    gh: torch.Tensor,
    h_in: torch.Tensor | None,
    h_out: torch.Tensor,
    w_s: torch.Tensor,
    z: torch.Tensor,
    alpha: torch.Tensor,
    s_scaled: torch.Tensor,
    *,
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """One small-batch Domino step: h_out = GRU gates(gi_table[tokens], gh, h_in), then
    s_scaled = bf16(alpha[0] * SiLU(z + bf16(w_s . h_out))) in the same launch
    (``tokens_are_keys`` as in :func:`gru_rank_gemv`)."""
    _require_cuda("tokens", tokens, torch.int64)
    for name, t in (("gi_table", gi_table), ("gh", gh), ("h_out", h_out), ("w_s", w_s), ("z", z)):
        _require_cuda(name, t, torch.bfloat16, 2)
    B, G = h_out.shape
    V = gi_table.shape[0]
    M = w_s.shape[0]
    if gh.shape != (B, 3 * G) or gh.stride(1) != 1 or gi_table.shape[1] != 3 * G or not h_out.is_contiguous():
        raise ValueError("GRU gate operands do not match the hidden size")
    if h_in is not None and (h_in.shape != (B, G) or not h_in.is_contiguous()):
        raise ValueError("h_in must be a contiguous [B, G] tensor")
    if w_s.shape[1] != G or z.shape != (B, M) or z.stride(1) != 1 or s_scaled.shape != (B, M) \
            or not s_scaled.is_contiguous():
        raise ValueError("correction MLP shapes do not match")
    tok_stride = tokens.stride(0) if tokens.dim() >= 1 and tokens.numel() > 1 else 1
    _lib.call("dels_gru_correction_mid_bf16", _ptr(tokens), tok_stride, int(tokens_are_keys), _ptr(gi_table),
              _row_major("gi_table", gi_table), _ptr(gh), gh.stride(0), _ptr(h_in), _ptr(h_out), B, G, V, _ptr(w_s),
              _row_major("w_s", w_s), _ptr(z), _row_major("z", z), M, _ptr(_f32_vec("alpha", alpha, h_out.device)),
              _ptr(s_scaled), _ptr(keys), None if ws is None else ws.ptr, _stream(h_out.device))
    return s_scaled


def rank_gemv(
    x: torch.Tensor,
    w: torch.Tensor,
    alpha: torch.Tensor | None,
    s_scaled: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    n_pos: int = 1,
    row_pos: torch.Tensor | None = None,
    activation: str = "identity",
    s_out: torch.Tensor | None = None,
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
) -> torch.Tensor:
    """Small-batch rank projection: s_scaled = bf16(alpha * act(x . w^T + bias))."""
    _require_cuda("x", x, torch.bfloat16, 2)
    _require_cuda("w", w, torch.bfloat16, 2)
    B, K = x.shape
    r = w.shape[0]
    if w.shape[1] != K or s_scaled.shape != (B, r) or not s_scaled.is_contiguous():
        raise ValueError("rank projection shapes do not match")
    _lib.call("dels_rank_gemv_bf16", _ptr(x), _row_major("x", x), _ptr(w), _row_major("w", w), _ptr(bias), B, K, r,
              ACTIVATIONS[activation], _ptr(alpha), int(n_pos), _ptr(_i32_vec("row_pos", row_pos)), _ptr(s_out),
              _ptr(s_scaled), _ptr(keys), None if ws is None else ws.ptr, _stream(x.device))
    return s_scaled


def gather_scaled_rows(
    tokens: torch.Tensor,
    emb: torch.Tensor,
    alpha: torch.Tensor | None,
    s_scaled: torch.Tensor,
    *,
    n_pos: int = 1,
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
    tokens_are_keys: bool = False,
) -> torch.Tensor:
    """s_scaled[b] = bf16(alpha * emb[tokens[b]]) (Markov rank state).  With
    ``tokens_are_keys`` the tokens are the previous step's packed (score, index) keys."""
    _require_cuda("tokens", tokens, torch.int64)
    _require_cuda("emb", emb, torch.bfloat16, 2)
    B, r = s_scaled.shape
    if emb.shape[1] != r or not s_scaled.is_contiguous():
        raise ValueError("embedding / output shapes do not match")
    tok_stride = tokens.stride(0) if tokens.numel() > 1 else 1
    _lib.call("dels_gather_scaled_rows_bf16", _ptr(tokens), tok_stride, int(bool(tokens_are_keys)), _ptr(emb),
              _row_major("emb", emb),
              _ptr(alpha), int(n_pos), B, r, emb.shape[0], _ptr(s_scaled), _ptr(keys),
              None if ws is None else ws.ptr, _stream(s_scaled.device))
    return s_scaled


def linear_workspace_bytes(rows: int, K: int, N: int) -> int:
    return int(_lib.query("dels_linear_workspace_bytes", rows, K, N))


def correction_mid_tc_workspace_bytes(B: int, G: int, M: int) -> int:
    return int(_lib.query("dels_correction_mid_tc_workspace_bytes", B, G, M))


def rank_workspace_bytes(rows: int, K: int, r: int) -> int:
    return int(_lib.query("dels_rank_workspace_bytes", rows, K, r))


def linear_bf16(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    out: torch.Tensor | None = None,
    ws: Workspace | None = None,
) -> torch.Tensor:
    """F.linear(x, w, bias) for bf16 operands: out = bf16(x . w^T + bias), one rounding."""
    _require_cuda("x", x, torch.bfloat16, 2)
    _require_cuda("w", w, torch.bfloat16, 2)
    rows, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w {tuple(w.shape)} does not match x {tuple(x.shape)}")
    if bias is not None:
        _require_cuda("bias", bias, torch.bfloat16, 1)
        if bias.shape[0] != N or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous [N] tensor")
    if out is None:
        out = torch.empty(rows, N, dtype=torch.bfloat16, device=x.device)
    elif out.shape != (rows, N) or out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise ValueError("out must be a row-major bf16 [rows, N] tensor")
    need = _lib.query("dels_linear_workspace_bytes", rows, K, N)
    ws = workspace(need, x.device) if ws is None else ws.ensure(need)
    _lib.call("dels_linear_bf16", _ptr(x), _row_major("x", x), _ptr(w), _row_major("w", w), _ptr(bias), rows, K, N,
              _ptr(out), _row_major("out", out), ws.ptr, ws.nbytes, _stream(x.device))
    return out


def correction_mid(
    h: torch.Tensor,
    w_s: torch.Tensor,
    z: torch.Tensor,
    alpha: torch.Tensor,
    s_scaled: torch.Tensor,
    *,
    keys: torch.Tensor | None = None,
    ws: Workspace | None = None,
) -> torch.Tensor:
    """Domino correction MLP hidden layer: s_scaled = bf16(alpha * SiLU(z + bf16(W_s h))), SiLU in fp32."""
    _require_cuda("h", h, torch.bfloat16, 2)
    _require_cuda("w_s", w_s, torch.bfloat16, 2)
    _require_cuda("z", z, torch.bfloat16, 2)
    B, G = h.shape
    M = w_s.shape[0]
    if w_s.shape[1] != G or z.shape != (B, M) or z.stride(1) != 1 or s_scaled.shape != (B, M) \
            or not s_scaled.is_contiguous():
        raise ValueError("correction MLP shapes do not match")
    _lib.call("dels_correction_mid_bf16", _ptr(h), _row_major("h", h), _ptr(w_s), _row_major("w_s", w_s), _ptr(z),
              _row_major("z", z), B, G, M, _ptr(alpha), _ptr(s_scaled), _ptr(keys),
              None if ws is None else ws.ptr, _stream(h.device))
    return s_scaled


def correction_mid_tc(
    h: torch.Tensor,
    w_s: torch.Tensor,
    z: torch.Tensor,
    alpha: torch.Tensor,
    s_scaled: torch.Tensor,
    *,
    keys: torch.Tensor | None = None,
    ws: Workspace,
) -> torch.Tensor:
    """correction_mid with W_s h on the tensor-core split-K GEMM (larger batches);
    ``ws`` needs correction_mid_tc_workspace_bytes(B, G, M)."""
    _require_cuda("h", h, torch.bfloat16, 2)
    _require_cuda("w_s", w_s, torch.bfloat16, 2)
    _require_cuda("z", z, torch.bfloat16, 2)
    B, G = h.shape
    M = w_s.shape[0]
    if w_s.shape[1] != G or z.shape != (B, M) or z.stride(1) != 1 or s_scaled.shape != (B, M) \
            or not s_scaled.is_contiguous():
        raise ValueError("correction MLP shapes do not match")
    _lib.call("dels_correction_mid_tc_bf16", _ptr(h), _row_major("h", h), _ptr(w_s), _row_major("w_s", w_s),
              _ptr(z), _row_major("z", z), B, G, M, _ptr(_f32_vec("alpha", alpha, h.device)), _ptr(s_scaled),
              _ptr(keys), ws.ptr, ws.nbytes, _stream(h.device))
    return s_scaled


def zero_pad(t: torch.Tensor | None, rows: int | None = None, cols: int | None = None) -> torch.Tensor | None:
    """``t`` zero-padded to ``rows`` (dim 0) x ``cols`` (dim 1).  The runners carry weight
    widths as multiples of 8 because TMA tiles need 16-byte row pitches; the zero entries
    contribute nothing to any contraction."""
    if t is None:
        return None
    shape = list(t.shape)
    if rows is not None:
        shape[0] = rows
    if cols is not None:
        shape[1] = cols
    if list(t.shape) == shape:
        return t
    out = torch.zeros(shape, dtype=t.dtype, device=t.device)
    out[tuple(slice(0, n) for n in t.shape)] = t
    return out


def round8(n: int) -> int:
    return -(-int(n) // 8) * 8
