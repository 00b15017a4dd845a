# coding=utf-8
"""DeLS local-head runtime helpers — drop-in for the reference's ``dels`` module.

Same public names, signatures, checkpoint formats and ``ValueError`` conditions as
code/dels.py: the unigram prior loader (:17-90), the alpha / beta schedule parser
(:93-112), the checkpoint-kind probe (:115-138) and the three local-head modules
(``DeLSLocalHead`` :141-345, ``MarkovDeLSLocalHead`` :348-430, ``PositionMixJointHead``
:433-621).  They load SpecForge checkpoints into modules whose weights the graph
runners in ``kernel/`` hand to the B200 kernels; the modules' own forward helpers
(``logits_from_hidden``, ``advance``) stay plain torch, as in the reference's eager path.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Iterable, Literal, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

_VALID_RANK_ACTIVATIONS = {"identity", "silu"}
_PRIOR_FILES = ("loss_mask_unigram.pt", "loss_mask_unigram.npz")


def _activation_check(rank_activation: str) -> None:
    if rank_activation not in _VALID_RANK_ACTIVATIONS:
        raise ValueError(f"rank_activation={rank_activation!r}; must be one of {_VALID_RANK_ACTIVATIONS}")


def _counts_from_pt(p: Path) -> torch.Tensor:
    payload = torch.load(p, map_location="cpu", weights_only=False)
    if torch.is_tensor(payload):
        return payload
    if isinstance(payload, dict) and "counts" in payload:
        return payload["counts"]
    raise ValueError(
        f"Unsupported unigram baseline .pt payload in {p}: expected a tensor or a dict with key 'counts'."
    )


def _counts_from_npz(p: Path) -> torch.Tensor:
    import numpy as np

    archive = np.load(p)
    if "counts" not in archive.files:
        raise ValueError(f"Unigram baseline npz {p} has no 'counts'.")
    return torch.from_numpy(archive["counts"])


# file suffix -> reader of the raw counts; a directory is resolved to the first of
# _PRIOR_FILES it holds
_COUNT_READERS = {".pt": _counts_from_pt, ".npz": _counts_from_npz}


def _read_counts(path: str) -> torch.Tensor:
    """Unigram counts (float64, flat) from a .pt / .npz file or a directory holding one."""
    p = Path(path)
    if p.is_dir():
        p = next((p / name for name in _PRIOR_FILES if (p / name).exists()), None)
        if p is None:
            raise ValueError(
                f"Unigram baseline directory {path!r} must contain loss_mask_unigram.pt or loss_mask_unigram.npz."
            )
    reader = _COUNT_READERS.get(p.suffix)
    if reader is None:
        raise ValueError(f"Unsupported unigram baseline path {p}; expected .pt, .npz, or a directory.")
    return reader(p).to(torch.float64).reshape(-1)


def load_unigram_log_prior(
    path: str,
    *,
    vocab_size: int,
    dtype: torch.dtype,
    device: torch.device,
    smoothing: float = 1.0,
) -> torch.Tensor:
    """Load a finite full-vocab log unigram prior as [1, 1, vocab_size].

    log((c + s) / sum(c + s)) computed in float64; counts shorter than the vocabulary
    are zero-padded; with s = 0 zero-count tokens get the smallest finite value."""
    if smoothing < 0:
        raise ValueError("smoothing must be non-negative.")
    counts = _read_counts(path)
    n = counts.numel()
    if n > vocab_size:
        raise ValueError(f"Unigram baseline vocab size {n} exceeds runtime vocab size {vocab_size}.")
    if n < vocab_size:
        counts = torch.cat([counts, counts.new_zeros(vocab_size - n)])
    if smoothing == 0.0:
        seen = counts > 0
        if not bool(seen.any()):
            raise ValueError("Unigram baseline has no positive counts.")
        logp = torch.full_like(counts, float("-inf"))
        logp[seen] = counts[seen].log() - counts.sum().log()
        logp[~seen] = logp[seen].min()
    else:
        shifted = counts + float(smoothing)
        logp = shifted.log() - shifted.sum().log()
    return logp.to(device=device, dtype=dtype).view(1, 1, vocab_size)


def parse_scalar_schedule(values: str | float | Iterable[float], steps: int, *, name: str) -> list[float]:
    """Parse a scalar or comma-separated per-position scalar schedule."""
    if isinstance(values, str):
        items = [float(tok.strip()) for tok in values.split(",") if tok.strip()]
    elif isinstance(values, (float, int)):
        items = [float(values)]
    else:
        items = [float(v) for v in values]
    if not items:
        raise ValueError(f"{name} schedule cannot be empty.")
    if len(items) == 1:
        return items * steps
    if len(items) != steps:
        raise ValueError(f"{name} schedule length must be 1 or {steps}, got {len(items)}.")
    return items


def _state(ckpt) -> dict | None:
    st = ckpt.get("model_state_dict")
    return st if isinstance(st, dict) else None


# Ordered probes: the first that matches names the runtime for a checkpoint.
_KIND_PROBES: tuple[tuple[Callable[[dict], bool], str], ...] = (
    (lambda ck: _state(ck) is not None and "down_proj" in _state(ck) and "up_proj" in _state(ck), "markov"),
    (lambda ck: _state(ck) is not None and any(k.startswith("prefix_gru.") for k in _state(ck)), "dels"),
    (lambda ck: isinstance(ck.get("model_config"), dict) and "gru_hidden_dim" in ck["model_config"], "dels"),
    (lambda ck: "embedding_weight" in ck and "lm_head_weight" in ck, "markov"),
)


def detect_local_head_checkpoint_kind(checkpoint_path: str) -> Literal["dels", "markov"]:
    """Return the local-head runtime kind for a SpecForge checkpoint."""
    ckpt = torch.load(checkpoint_path, map_location="cpu", weights_only=False)
    for matches, kind in _KIND_PROBES:
        if matches(ckpt):
            return kind  # type: ignore[return-value]
    raise ValueError(
        "Cannot identify local-head checkpoint type. Expected a SpecForge local_head.pt, "
        "merged_rnn_local_head.pt, markov_local_head.pt, or merged_markov_local_head.pt."
    )


# ----------------------------------------------------------------------------- state-dict schemas
# A checkpoint kind is described by a _Schema: how checkpoint keys map to module keys, an
# ordered list of rules (the first rule whose predicate accepts an entry decides what
# happens to it), which missing module keys are tolerated, and the error texts.  One
# routine, _apply_schema, walks any state dict with any schema.

def _open_checkpoint(path: str, what: str, checks) -> tuple[dict, dict]:
    """(model_config, model_state_dict) of a training checkpoint, after the kind's
    ordered (rejects(config, state), message) checks."""
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    config, state = ckpt.get("model_config"), ckpt.get("model_state_dict")
    if config is None or state is None:
        raise ValueError(f"{what} checkpoint must contain model_config and model_state_dict.")
    for rejects, message in checks:
        if rejects(config, state):
            raise ValueError(message)
    return config, state


_JOINT_CONFIG_CHECKS = (
    (lambda cfg, st: cfg.get("method") != "block_prefix_position_mix_joint",
     "Only block_prefix_position_mix_joint checkpoints are supported."),
    (lambda cfg, st: cfg.get("rnn_input", "block_prefix") != "block_prefix",
     "Only block_prefix position-joint checkpoints are supported."),
    (lambda cfg, st: cfg.get("local_head_config") is None, "Checkpoint is missing local_head_config."),
    (lambda cfg, st: "baseline_logits" not in st, "Block-prefix position checkpoint is missing baseline_logits."),
)

_FROZEN_PREFIXES = ("embed_tokens.", "target_lm_head.")  # tensors that belong to the target model


@dataclass
class _Entry:
    key: str  # key in the checkpoint
    name: Optional[str]  # module key it maps to (None: not one of the module's tensors)
    tensor: torch.Tensor


@dataclass(frozen=True)
class _Rule:
    """``applies(entry, own_state, ctx)``; ``action`` one of load / load_reshaped /
    frozen / fold_rank_to_hidden / reject (``message(entry, ctx)`` gives the text)."""

    applies: Callable[[_Entry, dict, dict], bool]
    action: str
    message: Optional[Callable[[_Entry, dict], str]] = None


@dataclass(frozen=True)
class _Schema:
    rename: Callable[[str], Optional[str]]
    rules: tuple[_Rule, ...]
    tolerated_missing: Callable[[str, nn.Module], bool]
    mismatch: Callable[[list, list, list], str]


def _shape_match(e: _Entry, own: dict, ctx: dict) -> bool:
    return e.name in own and own[e.name].shape == e.tensor.shape


def _apply_schema(model: nn.Module, state: dict, schema: _Schema, ctx: dict,
                  extra: Optional[dict] = None) -> None:
    """Load ``state`` into ``model`` as ``schema`` prescribes; ``extra`` entries (module
    key -> tensor) override the checkpoint's.  Raises ValueError with the schema's texts."""
    own = model.state_dict()
    plan: dict[str, torch.Tensor] = {}
    frozen: list[str] = []
    for key, tensor in state.items():
        e = _Entry(key, schema.rename(key), tensor)
        rule = next((r for r in schema.rules if r.applies(e, own, ctx)), None)
        if rule is None or rule.action == "reject":
            raise ValueError(rule.message(e, ctx) if rule is not None and rule.message else f"cannot load {key}")
        if rule.action == "load":
            plan[e.name] = tensor.to(dtype=own[e.name].dtype)
        elif rule.action == "load_reshaped":
            plan[e.name] = tensor.reshape_as(own[e.name]).to(dtype=own[e.name].dtype)
        elif rule.action == "fold_rank_to_hidden":
            w = own["low_rank_lm_head.weight"]
            plan["low_rank_lm_head.weight"] = (ctx["target_lm_head"].float() @ tensor.float()).to(dtype=w.dtype)
        else:  # frozen: owned by the target model, recorded for the error text
            frozen.append(key)
    for name, tensor in (extra or {}).items():
        plan[name] = tensor.to(dtype=own[name].dtype)
    missing, unexpected = model.load_state_dict(plan, strict=False)
    missing = [k for k in missing if not schema.tolerated_missing(k, model)]
    if missing or unexpected:
        raise ValueError(schema.mismatch(missing, unexpected, frozen))


def _dels_tolerated(key: str, model: nn.Module) -> bool:
    if key.startswith(_FROZEN_PREFIXES):
        return True
    unused = {"low_rank": "rank_to_hidden.", "target_lm_head": "low_rank_lm_head."}.get(model.lm_head_mode)
    return unused is not None and key.startswith(unused)


# DeLSLocalHead (local_head.pt, merged_rnn_local_head.pt): keys are module keys; a tensor
# of the module's shape loads; target-model tensors are skipped, except the embedding of
# a direct-vocab head, which is the head's own.
_DELS_SCHEMA = _Schema(
    rename=lambda key: key,
    rules=(
        _Rule(_shape_match, "load"),
        _Rule(lambda e, own, ctx: e.key.startswith(_FROZEN_PREFIXES)
              and not (ctx["direct_vocab"] and e.key.startswith("embed_tokens.")), "frozen"),
        _Rule(lambda e, own, ctx: True, "reject",
              lambda e, ctx: f"Unexpected local-head tensor {e.key} with shape {tuple(e.tensor.shape)}."),
    ),
    tolerated_missing=_dels_tolerated,
    mismatch=lambda m, u, f: f"Local-head checkpoint mismatch: missing={m}, unexpected={u}, skipped_frozen={f}",
)

_JOINT_PREFIX = "local_head_model."
_JOINT_TOP_LEVEL = ("position_gates", "baseline_logits")


def _joint_rename(key: str) -> Optional[str]:
    if key.startswith(_JOINT_PREFIX):
        return key[len(_JOINT_PREFIX):]
    return key if key in _JOINT_TOP_LEVEL else None


# PositionMixJointHead: the local head's tensors sit under "local_head_model.", the gates
# and the baseline at the top level; other keys (optimizer, target copies) are skipped; a
# rank_to_hidden projection is folded into the low-rank head when the local head used
# the target's LM head.
_JOINT_SCHEMA = _Schema(
    rename=_joint_rename,
    rules=(
        _Rule(lambda e, own, ctx: e.name is None or e.name.startswith(_FROZEN_PREFIXES), "frozen"),
        _Rule(lambda e, own, ctx: e.name == "baseline_logits", "load_reshaped"),
        _Rule(_shape_match, "load"),
        _Rule(lambda e, own, ctx: e.name == "rank_to_hidden.weight" and ctx["lm_head_mode"] != "target_lm_head",
              "reject",
              lambda e, ctx: "Unexpected rank_to_hidden.weight for block-prefix joint local "
                             f"lm_head_mode={ctx['lm_head_mode']!r}."),
        _Rule(lambda e, own, ctx: e.name == "rank_to_hidden.weight", "fold_rank_to_hidden"),
        _Rule(lambda e, own, ctx: True, "reject",
              lambda e, ctx: f"Unexpected block-prefix joint tensor {e.key} mapped to {e.name} with shape "
                             f"{tuple(e.tensor.shape)}."),
    ),
    tolerated_missing=lambda key, model: key.startswith(_FROZEN_PREFIXES),
    mismatch=lambda m, u, f: f"Block-prefix position checkpoint mismatch: missing={m}, unexpected={u}, skipped={f}",
)


def _rank_logits(module, hidden: torch.Tensor) -> torch.Tensor:
    """low_rank_lm_head(act(rank_proj(hidden^T))) for hidden [1, B, G]."""
    rank_state = module.rank_proj(hidden.transpose(0, 1))
    if module.rank_activation == "silu":
        rank_state = F.silu(rank_state)
    return module.low_rank_lm_head(rank_state)


def _gru(embed_dim: int, hidden: int) -> nn.GRU:
    return nn.GRU(input_size=embed_dim, hidden_size=hidden, num_layers=1, batch_first=True, bias=False)


class DeLSLocalHead(nn.Module):
    """Inference module for SpecForge local-head checkpoints (bias-free GRU over the
    block's chosen tokens -> rank projection -> low-rank LM head)."""

    def __init__(
        self,
        *,
        target_model: nn.Module,
        vocab_size: int,
        embed_dim: int,
        gru_hidden_dim: int,
        low_rank_dim: int,
        lm_head_mode: str,
        rank_activation: str = "identity",
        dtype: torch.dtype,
        device: torch.device,
        target_lm_head: Optional[nn.Module] = None,
        embedding_weight: Optional[torch.Tensor] = None,
    ):
        super().__init__()
        _activation_check(rank_activation)
        if embedding_weight is None:
            self.embed_tokens = target_model.model.embed_tokens
        else:
            want = (int(vocab_size), int(embed_dim))
            if tuple(embedding_weight.shape) != want:
                raise ValueError(f"Local embedding shape {tuple(embedding_weight.shape)} does not match config {want}.")
            if target_model.lm_head.weight.shape[0] != int(vocab_size):
                raise ValueError("Local-head vocabulary does not match the target model.")
            self.embed_tokens = nn.Embedding.from_pretrained(embedding_weight.to(device=device, dtype=dtype),
                                                             freeze=True)
        self.vocab_size = int(vocab_size)
        self.embed_dim = int(embed_dim)
        self.gru_hidden_dim = int(gru_hidden_dim)
        self.low_rank_dim = int(low_rank_dim)
        self.lm_head_mode = lm_head_mode
        self.rank_activation = rank_activation
        self.prefix_gru = _gru(self.embed_dim, self.gru_hidden_dim)
        self.rank_proj = nn.Linear(self.gru_hidden_dim, self.low_rank_dim, bias=False)
        self.low_rank_lm_head = nn.Linear(self.low_rank_dim, self.vocab_size, bias=False)
        self.rank_to_hidden = None
        self.target_lm_head = None
        if lm_head_mode == "target_lm_head":
            if target_lm_head is None:
                raise ValueError("target_lm_head is required for target_lm_head mode.")
            self.rank_to_hidden = nn.Linear(self.low_rank_dim, int(target_lm_head.weight.shape[1]), bias=False)
            self.target_lm_head = target_lm_head
        self.to(device=device, dtype=dtype)
        self.eval()

    @classmethod
    def from_checkpoint(
        cls,
        *,
        checkpoint_path: str,
        target_model: nn.Module,
        dtype: torch.dtype,
        device: torch.device,
        merged_lm_head_path: Optional[str] = None,
    ) -> "DeLSLocalHead":
        config, state = _open_checkpoint(checkpoint_path, "Local-head", ())
        param = config.get("rnn_parameterization", config.get("local_head_parameterization"))
        direct_vocab = param == "direct_vocab" or config.get("architecture") == "direct_vocab_rnn"
        embedding_weight = None
        if direct_vocab:
            embedding_weight = state.get("embed_tokens.weight")
            if embedding_weight is None:
                raise ValueError("Direct-vocab RNN checkpoint has no embed_tokens.weight.")
        elif "embed_down_proj.weight" in state:
            raise ValueError(
                "This RNN checkpoint has an input projection. Use merged_rnn_local_head.pt or convert it with "
                "SpecForge scripts/convert_local_head.py before inference."
            )
        model = cls(
            target_model=target_model,
            vocab_size=int(config["vocab_size"]),
            embed_dim=int(config["embed_dim"]),
            gru_hidden_dim=int(config["gru_hidden_dim"]),
            low_rank_dim=int(config["low_rank_dim"]),
            lm_head_mode=config.get("lm_head_mode", "low_rank"),
            rank_activation=config.get("rank_activation", "identity"),
            dtype=dtype,
            device=device,
            target_lm_head=target_model.lm_head,
            embedding_weight=embedding_weight,
        )
        model.pure_draft_prefix_len = int(config.get("pure_draft_prefix_len", 0 if direct_vocab else 1))
        model.shift_label = bool(config.get("shift_label", False))
        extra = None
        if merged_lm_head_path is not None:
            merged = torch.load(merged_lm_head_path, map_location="cpu", weights_only=False)
            extra = {"low_rank_lm_head.weight": merged["weight"] if isinstance(merged, dict) else merged}
            model.lm_head_mode = "low_rank"
        _apply_schema(model, state, _DELS_SCHEMA, {"direct_vocab": direct_vocab}, extra)
        if model.lm_head_mode == "target_lm_head":
            model.fuse_target_lm_head_()
        return model

    @torch.inference_mode()
    def fuse_target_lm_head_(self) -> None:
        """Fold target_lm_head . rank_to_hidden into low_rank_lm_head (fp32 product)."""
        if self.lm_head_mode != "target_lm_head":
            return
        if self.rank_to_hidden is None or self.target_lm_head is None:
            raise ValueError("Cannot fuse local head without rank_to_hidden/target_lm_head.")
        fused = self.target_lm_head.weight.detach().float() @ self.rank_to_hidden.weight.detach().float()
        self.low_rank_lm_head.weight.copy_(fused.to(self.low_rank_lm_head.weight.dtype))
        self.rank_to_hidden = None
        self.target_lm_head = None
        self.lm_head_mode = "low_rank"

    @torch.inference_mode()
    def init_empty_hidden(self, batch_size: int, *, device: torch.device) -> torch.Tensor:
        return torch.zeros(1, batch_size, self.gru_hidden_dim, device=device, dtype=self.rank_proj.weight.dtype)

    @torch.inference_mode()
    def logits_from_hidden(self, hidden: torch.Tensor) -> torch.Tensor:
        return _rank_logits(self, hidden)

    @torch.inference_mode()
    def advance(self, token_ids: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
        _, hidden = self.prefix_gru(self.embed_tokens(token_ids), hidden)
        return hidden


def _markov_merged(ckpt: dict, target_model) -> tuple[torch.Tensor, torch.Tensor]:
    return ckpt["embedding_weight"], ckpt["lm_head_weight"]


def _markov_factorized(ckpt: dict, target_model) -> tuple[torch.Tensor, torch.Tensor]:
    """embedding = E_target . down, lm_head = W_target . up^T (fp32 products)."""
    config, state = ckpt.get("model_config"), ckpt.get("model_state_dict")
    if config is None or state is None:
        raise ValueError(
            "Markov DeLS checkpoint must be either merged_markov_local_head.pt or markov_local_head.pt "
            "from SpecForge scripts/train_markov_local_head.py."
        )
    if "down_proj" not in state or "up_proj" not in state:
        raise ValueError("Markov local-head checkpoint must contain down_proj and up_proj.")
    down, up = state["down_proj"].to(torch.float32), state["up_proj"].to(torch.float32)
    emb = target_model.model.embed_tokens.weight.detach().cpu().to(torch.float32) @ down
    head = target_model.lm_head.weight.detach().cpu().to(torch.float32) @ up.t()
    want_rank = int(config.get("rank", down.shape[1]))
    if emb.shape[1] != want_rank:
        raise ValueError(f"Unexpected Markov rank: merged={emb.shape[1]}, config={want_rank}")
    return emb, head


# Ordered (accepts, factors) pairs: merged_markov_local_head.pt carries both merged
# factors; anything else is read as the factorised training checkpoint.
_MARKOV_FORMATS: tuple[tuple[Callable[[dict], bool], Callable], ...] = (
    (lambda ck: "embedding_weight" in ck and "lm_head_weight" in ck, _markov_merged),
    (lambda ck: True, _markov_factorized),
)


class MarkovDeLSLocalHead(nn.Module):
    """Inference module for dense Markov local-head checkpoints: logits of the next token
    are embedding[prev] . lm_head^T with both factors merged to the vocabulary."""

    def __init__(self, *, embedding_weight: torch.Tensor, lm_head_weight: torch.Tensor, dtype: torch.dtype,
                 device: torch.device):
        super().__init__()
        if embedding_weight.ndim != 2 or lm_head_weight.ndim != 2:
            raise ValueError("Markov DeLS weights must be rank-2 tensors.")
        if embedding_weight.shape[1] != lm_head_weight.shape[1]:
            raise ValueError(
                "Markov DeLS merged embedding/lm-head rank mismatch: "
                f"embedding={tuple(embedding_weight.shape)}, lm_head={tuple(lm_head_weight.shape)}"
            )
        self.embedding_weight = nn.Parameter(embedding_weight.to(device=device, dtype=dtype), requires_grad=False)
        self.lm_head_weight = nn.Parameter(lm_head_weight.to(device=device, dtype=dtype), requires_grad=False)
        self.vocab_size = int(lm_head_weight.shape[0])
        self.rank = int(lm_head_weight.shape[1])
        self.eval()

    @classmethod
    def from_checkpoint(cls, *, checkpoint_path: str, target_model: nn.Module, dtype: torch.dtype,
                        device: torch.device) -> "MarkovDeLSLocalHead":
        ckpt = torch.load(checkpoint_path, map_location="cpu", weights_only=False)
        for matches, factors in _MARKOV_FORMATS:
            if matches(ckpt):
                emb, head = factors(ckpt, target_model)
                return cls(embedding_weight=emb, lm_head_weight=head, dtype=dtype, device=device)
        raise AssertionError("unreachable: the last Markov format accepts every checkpoint")

    @torch.inference_mode()
    def logits_from_token(self, token_ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(token_ids, self.embedding_weight) @ self.lm_head_weight.t()


class PositionMixJointHead(nn.Module):
    """Runtime for block-prefix position joint finetune checkpoints: a DeLS local head
    plus per-suffix-position (alpha, beta) gates and its own baseline logits."""

    def __init__(
        self,
        *,
        target_model: nn.Module,
        vocab_size: int,
        embed_dim: int,
        gru_hidden_dim: int,
        low_rank_dim: int,
        suffix_len: int,
        shift_label: bool,
        rank_activation: str,
        baseline_logits: torch.Tensor,
        dtype: torch.dtype,
        device: torch.device,
    ):
        super().__init__()
        _activation_check(rank_activation)
        self.embed_tokens = target_model.model.embed_tokens
        self.vocab_size = int(vocab_size)
        self.embed_dim = int(embed_dim)
        self.gru_hidden_dim = int(gru_hidden_dim)
        self.low_rank_dim = int(low_rank_dim)
        self.pure_draft_prefix_len = 1
        self.shift_label = bool(shift_label)
        self.rank_activation = rank_activation
        self.rnn_input = "block_prefix"
        self.mix_form = "block_prefix_position"
        self.prefix_gru = _gru(self.embed_dim, self.gru_hidden_dim)
        self.rank_proj = nn.Linear(self.gru_hidden_dim, self.low_rank_dim, bias=False)
        self.low_rank_lm_head = nn.Linear(self.low_rank_dim, self.vocab_size, bias=False)
        self.position_gates = nn.Parameter(torch.zeros(int(suffix_len), 2, dtype=dtype, device=device))
        self.register_buffer("baseline_logits", baseline_logits.to(device=device, dtype=dtype).view(1, 1, -1),
                             persistent=True)
        self.to(device=device, dtype=dtype)
        self.eval()

    @classmethod
    def from_checkpoint(cls, *, checkpoint_path: str, target_model: nn.Module, block_size: int,
                        dtype: torch.dtype, device: torch.device) -> "PositionMixJointHead":
        config, state = _open_checkpoint(checkpoint_path, "Block-prefix position", _JOINT_CONFIG_CHECKS)
        local = config["local_head_config"]
        shift_label = bool(config.get("dflash_shift_label", False))
        suffix_len = int(block_size) - (1 if shift_label else 2)
        if suffix_len <= 0:
            raise ValueError(
                "Block-prefix position checkpoint has no suffix positions: "
                f"block_size={block_size}, suffix_start={1 if shift_label else 2}."
            )
        model = cls(
            target_model=target_model,
            vocab_size=int(local["vocab_size"]),
            embed_dim=int(local["embed_dim"]),
            gru_hidden_dim=int(local["gru_hidden_dim"]),
            low_rank_dim=int(local["low_rank_dim"]),
            suffix_len=suffix_len,
            shift_label=shift_label,
            rank_activation=local.get("rank_activation", "identity"),
            baseline_logits=state["baseline_logits"],
            dtype=dtype,
            device=device,
        )
        ctx = {"lm_head_mode": local.get("lm_head_mode", "low_rank"),
               "target_lm_head": target_model.lm_head.weight.detach()}
        _apply_schema(model, state, _JOINT_SCHEMA, ctx)
        return model

    @torch.inference_mode()
    def init_empty_hidden(self, batch_size: int, *, device: torch.device) -> torch.Tensor:
        return torch.zeros(1, batch_size, self.gru_hidden_dim, device=device, dtype=self.rank_proj.weight.dtype)

    @torch.inference_mode()
    def logits_from_hidden(self, hidden: torch.Tensor) -> torch.Tensor:
        return _rank_logits(self, hidden)

    @torch.inference_mode()
    def alpha_beta_schedules(self) -> tuple[list[float], list[float]]:
        gates = self.position_gates.detach().to(device="cpu", dtype=torch.float32)
        return gates[:, 0].tolist(), gates[:, 1].tolist()

    @torch.inference_mode()
    def advance(self, token_ids: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
        _, hidden = self.prefix_gru(self.embed_tokens(token_ids), hidden)
        return hidden
