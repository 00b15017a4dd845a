"""Generate the golden fixtures in this directory by running the REFERENCE's own code.

Usage (needs a checkout of the reference; it is not available on GPU machines, which
only read the committed fixtures):

    python tests/golden/make_golden.py --reference <reference checkout>/code

What runs, and from where in the reference:
  * ``dels.parse_scalar_schedule`` (code/dels.py:93-112) on a table of inputs;
  * ``dels.load_unigram_log_prior`` (code/dels.py:17-90) on synthetic ``counts`` files
    (.pt dict / .pt tensor / .npz, padded, smoothing 1, 0.5 and 0);
  * the scorer: ``dels.DeLSLocalHead.logits_from_hidden`` (code/dels.py:334-339) for the
    low-rank logits, an ``nn.Linear`` target LM head for the long logits
    (code/dflash.py:468), the mix of code/dflash.py:523-527 and ``dflash.sample``
    (code/dflash.py:31-33) for the argmax — in fp32 and in bf16;
  * ``kernel.dels.DeLSGraphRunner`` (code/kernel/dels.py:214-478) and
    ``kernel.markov_dels.MarkovDeLSGraphRunner`` (code/kernel/markov_dels.py:139-312)
    end to end on the CPU: their CUDA stream / graph calls are replaced by stand-ins
    that run the captured function eagerly, and the Triton kernels are disabled, so the
    runners execute their own torch fallback path (code/kernel/dels.py:447-456);
  * ``kernel.domino.DraftCorrectionGraphRunner`` (code/kernel/domino.py:232-520) on the CPU
    the same way: its torch path in fp32 and bf16 (Triton disabled), and its fused
    Triton step (code/kernel/domino.py:57-229) run by Triton's CPU interpreter in bf16;
  * the acceptance expression of code/dflash.py:645-651, evaluated with torch exactly as
    written there;
  * the checkpoint loaders of code/dels.py (``detect_local_head_checkpoint_kind``,
    ``DeLSLocalHead.from_checkpoint`` incl. target-LM-head fusion and merged heads,
    ``MarkovDeLSLocalHead.from_checkpoint``, ``PositionMixJointHead.from_checkpoint``) on
    small synthetic SpecForge-style checkpoints written to ``ckpt/``.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent


def bf16_values(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).cpu().numpy()


class _FakeStream:
    def wait_stream(self, other):
        return None


class _FakeGraph:
    def __init__(self):
        self.replay = lambda: None


@contextlib.contextmanager
def cpu_graph_standins():
    """Let the reference runners construct and replay on the CPU."""
    saved = {k: getattr(torch.cuda, k) for k in ("Stream", "current_stream", "stream", "CUDAGraph", "graph")}
    torch.cuda.Stream = lambda *a, **k: _FakeStream()
    torch.cuda.current_stream = lambda *a, **k: _FakeStream()
    torch.cuda.stream = lambda *a, **k: contextlib.nullcontext()
    torch.cuda.CUDAGraph = _FakeGraph
    torch.cuda.graph = lambda *a, **k: contextlib.nullcontext()
    try:
        yield
    finally:
        for k, v in saved.items():
            setattr(torch.cuda, k, v)


def stub_target(V: int, E: int, H: int, dtype) -> types.SimpleNamespace:
    model = types.SimpleNamespace(embed_tokens=nn.Embedding(V, E).to(dtype))
    return types.SimpleNamespace(model=model, lm_head=nn.Linear(H, V, bias=False).to(dtype))


# ------------------------------------------------------------------------------ schedules
def gen_schedules(ref) -> None:
    cases = [
        ("0.3", 4),
        (0.5, 3),
        (2, 2),
        ("0.5, 0.4,0.3", 3),
        ("1,", 5),
        ([0.1, 0.2], 2),
        ("", 3),
        ("0.1,0.2", 3),
        ([], 2),
        ((0.7,), 4),
    ]
    out = []
    for values, steps in cases:
        try:
            res = {"ok": ref.dels.parse_scalar_schedule(values, steps, name="DeLS alpha")}
        except ValueError as exc:
            res = {"error": str(exc)}
        out.append({"values": values if not isinstance(values, tuple) else list(values), "is_tuple": isinstance(values, tuple), "steps": steps, **res})
    (HERE / "schedules.json").write_text(json.dumps(out, indent=1) + "\n")


# ------------------------------------------------------------------------------ priors
def gen_priors(ref) -> None:
    rng = np.random.default_rng(11)
    V = 777
    counts = rng.integers(0, 50, size=700).astype(np.float64)
    counts[::7] = 0
    arrays = {"counts": counts, "vocab_size": np.array(V)}
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        torch.save({"counts": torch.from_numpy(counts)}, td / "dict.pt")
        torch.save(torch.from_numpy(counts), td / "tensor.pt")
        np.savez(td / "c.npz", counts=counts)
        sub = td / "dir"
        sub.mkdir()
        np.savez(sub / "loss_mask_unigram.npz", counts=counts)
        for tag, path in (("dict_pt", "dict.pt"), ("tensor_pt", "tensor.pt"), ("npz", "c.npz"), ("dir", "dir")):
            for sm in (1.0, 0.5, 0.0):
                for dtype, dname in ((torch.float64, "f64"), (torch.bfloat16, "bf16")):
                    lp = ref.dels.load_unigram_log_prior(
                        str(td / path), vocab_size=V, dtype=dtype, device=torch.device("cpu"), smoothing=sm
                    )
                    arrays[f"{tag}_s{sm}_{dname}"] = lp.to(torch.float64).reshape(-1).numpy()
    np.savez_compressed(HERE / "priors.npz", **arrays)


# ------------------------------------------------------------------------------ scorer
def gen_scorer(ref) -> None:
    arrays: dict[str, np.ndarray] = {}
    cases = [
        # name, seed, B, P, H, r, V, activation, with_prior
        ("a", 0, 2, 8, 96, 24, 1000, "identity", True),
        ("b", 1, 3, 5, 64, 16, 1031, "silu", True),
        ("c", 2, 1, 16, 128, 32, 517, "identity", False),
    ]
    meta = []
    for name, seed, B, P, H, r, V, act, with_prior in cases:
        g = torch.Generator().manual_seed(seed)
        rows = B * P
        h = bf16_values(torch.randn(rows, H, generator=g))
        W = bf16_values(torch.randn(V, H, generator=g) * 0.05)
        Ut = bf16_values(torch.randn(r, H, generator=g) * 0.05)
        Vr = bf16_values(torch.randn(V, r, generator=g) * 0.1)
        alpha = [round(0.5 - 0.4 * p / max(P - 1, 1), 4) for p in range(P)]
        beta = [round(0.3 - 0.3 * p / max(P - 1, 1), 4) for p in range(P)]
        counts = torch.randint(0, 1000, (V,), generator=g).to(torch.float64)
        arrays[f"{name}_h"] = f32(h)
        arrays[f"{name}_W"] = f32(W)
        arrays[f"{name}_Ut"] = f32(Ut)
        arrays[f"{name}_Vr"] = f32(Vr)
        arrays[f"{name}_alpha"] = np.array(alpha, np.float64)
        arrays[f"{name}_beta"] = np.array(beta, np.float64)
        for dtype, dname in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            target = stub_target(V, 8, H, dtype)
            head = ref.dels.DeLSLocalHead(
                target_model=target, vocab_size=V, embed_dim=8, gru_hidden_dim=H, low_rank_dim=r,
                lm_head_mode="low_rank", rank_activation=act, dtype=dtype, device=torch.device("cpu"),
            )
            with torch.no_grad():
                head.rank_proj.weight.copy_(Ut.to(dtype))
                head.low_rank_lm_head.weight.copy_(Vr.to(dtype))
                target.lm_head.weight.copy_(W.to(dtype))
            prior = None
            if with_prior:
                with tempfile.TemporaryDirectory() as td:
                    torch.save({"counts": counts}, Path(td) / "loss_mask_unigram.pt")
                    prior = ref.dels.load_unigram_log_prior(
                        td, vocab_size=V, dtype=dtype, device=torch.device("cpu")
                    )
                arrays[f"{name}_prior_{dname}"] = f32(prior.reshape(-1))
            x = h.to(dtype)
            with torch.inference_mode():
                long_logits = target.lm_head(x).view(B, P, V)
                short = head.logits_from_hidden(x.view(1, rows, H)).view(B, P, V)
                tokens = torch.empty(B, P, dtype=torch.long)
                final_all = torch.empty(B, P, V, dtype=torch.float32)
                for p in range(P):
                    long_p = long_logits[:, p : p + 1, :]
                    short_p = short[:, p : p + 1, :]
                    # the mix of code/dflash.py:523-527, as written there
                    final_logits = long_p + alpha[p] * short_p
                    if prior is not None:
                        final_logits = final_logits - beta[p] * prior
                    tokens[:, p] = ref.dflash.sample(final_logits)[:, 0]
                    final_all[:, p] = final_logits[:, 0].to(torch.float32)
            arrays[f"{name}_tokens_{dname}"] = tokens.reshape(-1).numpy()
            arrays[f"{name}_final_{dname}"] = final_all.reshape(rows, V).numpy()
        meta.append({"name": name, "B": B, "P": P, "H": H, "r": r, "V": V, "activation": act, "prior": with_prior})
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "scorer.npz", **arrays)


# ------------------------------------------------------------------------------ runners
def gen_runners(ref) -> None:
    ref.kernel_dels.HAS_TRITON = False
    ref.kernel_markov.HAS_TRITON = False
    arrays: dict[str, np.ndarray] = {}
    meta = []
    cases = [
        # name, seed, B, steps, V, E, G, r, activation, with_prior
        ("g1", 5, 3, 6, 1000, 32, 64, 16, "identity", True),
        ("g2", 6, 2, 14, 611, 24, 48, 32, "silu", True),
        ("g3", 7, 1, 4, 300, 16, 32, 8, "identity", False),
    ]
    for name, seed, B, steps, V, E, G, r, act, with_prior in cases:
        g = torch.Generator().manual_seed(seed)
        embed = bf16_values(torch.randn(V, E, generator=g) * 0.5)
        w_ih = bf16_values(torch.randn(3 * G, E, generator=g) * 0.2)
        w_hh = bf16_values(torch.randn(3 * G, G, generator=g) * 0.2)
        w_rank = bf16_values(torch.randn(r, G, generator=g) * 0.3)
        Vr = bf16_values(torch.randn(V, r, generator=g) * 0.3)
        base = bf16_values(torch.randn(B, steps, V, generator=g))
        prefix = torch.randint(0, V, (B, 1), generator=g)
        alpha = [round(0.9 - 0.05 * i, 4) for i in range(steps)]
        beta = [round(0.2 + 0.02 * i, 4) for i in range(steps)] if with_prior else [0.0] * steps
        counts = torch.randint(0, 500, (V,), generator=g).to(torch.float64)
        for k, v in (("embed", embed), ("w_ih", w_ih), ("w_hh", w_hh), ("w_rank", w_rank), ("Vr", Vr), ("base", base)):
            arrays[f"{name}_{k}"] = f32(v)
        arrays[f"{name}_prefix"] = prefix.numpy()
        arrays[f"{name}_alpha"] = np.array(alpha)
        arrays[f"{name}_beta"] = np.array(beta)
        for dtype, dname in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            target = stub_target(V, E, G, dtype)
            head = ref.dels.DeLSLocalHead(
                target_model=target, vocab_size=V, embed_dim=E, gru_hidden_dim=G, low_rank_dim=r,
                lm_head_mode="low_rank", rank_activation=act, dtype=dtype, device=torch.device("cpu"),
            )
            with torch.no_grad():
                head.embed_tokens.weight.copy_(embed.to(dtype))
                head.prefix_gru.weight_ih_l0.copy_(w_ih.to(dtype))
                head.prefix_gru.weight_hh_l0.copy_(w_hh.to(dtype))
                head.rank_proj.weight.copy_(w_rank.to(dtype))
                head.low_rank_lm_head.weight.copy_(Vr.to(dtype))
            prior = None
            if with_prior:
                with tempfile.TemporaryDirectory() as td:
                    torch.save({"counts": counts}, Path(td) / "loss_mask_unigram.pt")
                    prior = ref.dels.load_unigram_log_prior(td, vocab_size=V, dtype=dtype, device=torch.device("cpu"))
                arrays[f"{name}_prior_{dname}"] = f32(prior.reshape(-1))
            with cpu_graph_standins():
                runner = ref.kernel_dels.DeLSGraphRunner(
                    local_head=head, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                    beta_values=beta, baseline_logits=prior, device=torch.device("cpu"),
                )
            runner.graph.replay = runner._forward_impl
            out = runner(prefix, base.to(dtype))
            arrays[f"{name}_tokens_{dname}"] = out.numpy()
            # Markov runner on the same shapes: embedding rows are the rank states.
            emb_r = bf16_values(torch.randn(V, r, generator=torch.Generator().manual_seed(seed + 100)) * 0.5)
            arrays[f"{name}_markov_embedding"] = f32(emb_r)
            mhead = ref.dels.MarkovDeLSLocalHead(
                embedding_weight=emb_r.to(dtype), lm_head_weight=Vr.to(dtype), dtype=dtype,
                device=torch.device("cpu"),
            )
            with cpu_graph_standins():
                mrunner = ref.kernel_markov.MarkovDeLSGraphRunner(
                    local_head=mhead, batch_size=B, steps=steps, vocab_size=V, alpha_values=alpha,
                    beta_values=beta, baseline_logits=prior, device=torch.device("cpu"),
                )
            mrunner.graph.replay = mrunner._forward_impl
            arrays[f"{name}_markov_tokens_{dname}"] = mrunner(prefix, base.to(dtype)).numpy()
        meta.append({"name": name, "B": B, "steps": steps, "V": V, "E": E, "G": G, "r": r, "activation": act,
                     "prior": with_prior})
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "runners.npz", **arrays)


# ------------------------------------------------------------------------------ Domino
class _DominoDraft(nn.Module):
    """The Domino correction parts of the reference draft model (code/dflash.py:262-276)."""

    def __init__(self, H: int, G: int, M: int, V: int, bias: bool):
        super().__init__()
        self.prefix_gru = nn.GRU(input_size=H, hidden_size=G, num_layers=1, batch_first=True, bias=bias)
        self.embed_proj = nn.Sequential(nn.Linear(H + G, M, bias=bias), nn.SiLU(), nn.Linear(M, V, bias=bias))


DOMINO_CASES = [
    # name, seed, B, steps, prefix tokens, V, H, G, M, biases, alpha
    ("d1", 21, 2, 5, 2, 700, 48, 32, 24, True, 0.8),
    ("d2", 22, 1, 6, 1, 500, 32, 16, 40, False, 1.0),
    ("d3", 23, 3, 4, 3, 333, 40, 24, 16, True, 1.5),
]


def _domino_inputs(seed, B, steps, P, V, H, G, M, bias):
    g = torch.Generator().manual_seed(seed)
    draft = _DominoDraft(H, G, M, V, bias)
    with torch.no_grad():
        for prm in draft.parameters():
            prm.copy_(bf16_values(torch.randn(prm.shape, generator=g) * 0.3))
    embed = bf16_values(torch.randn(V, H, generator=g) * 0.5)
    hiddens = bf16_values(torch.randn(B, steps, H, generator=g))
    base = bf16_values(torch.randn(B, steps, V, generator=g))
    prefix = torch.randint(0, V, (B, P), generator=g)
    return draft, embed, hiddens, base, prefix


def _domino_run(module, case, dtype):
    name, seed, B, steps, P, V, H, G, M, bias, alpha = case
    draft, embed, hiddens, base, prefix = _domino_inputs(seed, B, steps, P, V, H, G, M, bias)
    draft = draft.to(dtype)
    target = types.SimpleNamespace(model=types.SimpleNamespace(embed_tokens=nn.Embedding(V, H)))
    with torch.no_grad():
        target.model.embed_tokens.weight.copy_(embed)
    target.model.embed_tokens = target.model.embed_tokens.to(dtype)
    with cpu_graph_standins():
        runner = module.DraftCorrectionGraphRunner(
            draft_model=draft, target_model=target, batch_size=B, steps=steps, hidden_dim=H, gru_hidden_dim=G,
            vocab_size=V, prefix_token_count=P, device=torch.device("cpu"), guidance_alpha=alpha,
        )
    runner.graph.replay = runner._forward_impl
    return runner(prefix, hiddens.to(dtype), base.to(dtype), alpha).numpy(), runner._can_triton_fuse


def domino_fused_worker(out_path: str) -> None:
    """Run in a process started with TRITON_INTERPRET=1 (the interpreter must be chosen
    before triton is first imported): the fused Triton step on the CPU, bf16."""
    import kernel.domino as interp  # noqa: E402

    arrays = {}
    for case in DOMINO_CASES:
        tokens, fused = _domino_run(interp, case, torch.bfloat16)
        assert fused, "the Triton path was not taken"
        arrays[f"{case[0]}_tokens_bf16_fused"] = tokens
    np.savez(out_path, **arrays)


def gen_domino(ref, reference_dir: Path) -> None:
    import os
    import subprocess

    arrays: dict[str, np.ndarray] = {}
    meta = []
    ref.kernel_domino.HAS_TRITON = False
    for case in DOMINO_CASES:
        name, seed, B, steps, P, V, H, G, M, bias, alpha = case
        draft, embed, hiddens, base, prefix = _domino_inputs(seed, B, steps, P, V, H, G, M, bias)
        for k, t in (("embed", embed), ("hiddens", hiddens), ("base", base)):
            arrays[f"{name}_{k}"] = f32(t)
        arrays[f"{name}_prefix"] = prefix.numpy()
        for k, t in draft.named_parameters():
            arrays[f"{name}_{k.replace('.', '_')}"] = f32(t)
        for dtype, dname in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            arrays[f"{name}_tokens_{dname}"], fused = _domino_run(ref.kernel_domino, case, dtype)
            assert not fused
        meta.append({"name": name, "B": B, "steps": steps, "P": P, "V": V, "H": H, "G": G, "M": M, "bias": bias,
                     "alpha": alpha})
    with tempfile.TemporaryDirectory() as td:
        out = Path(td) / "fused.npz"
        subprocess.run([sys.executable, str(Path(__file__).resolve()), "--reference", str(reference_dir),
                        "--domino-fused-worker", str(out)], check=True, env={**os.environ, "TRITON_INTERPRET": "1"})
        with np.load(out) as f:
            for k in f.files:
                arrays[k] = f[k]
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "domino.npz", **arrays)


# ------------------------------------------------------------------------------ acceptance
def gen_accept() -> None:
    g = torch.Generator().manual_seed(2)
    n_seq, P, V = 64, 16, 50
    verify = torch.randint(0, V, (n_seq, P + 1), generator=g)
    posterior = torch.randint(0, V, (n_seq, P + 1), generator=g)
    k = torch.randint(0, P + 1, (n_seq,), generator=g)
    for b in range(n_seq):
        verify[b, 1 : 1 + int(k[b])] = posterior[b, : int(k[b])]
    # code/dflash.py:646-651, as written there (batched over sequences)
    acceptance_length = (verify[:, 1:] == posterior[:, :-1]).cumprod(dim=1).sum(dim=1)
    np.savez_compressed(
        HERE / "accept.npz", verify=verify.numpy(), posterior=posterior.numpy(), accept=acceptance_length.numpy()
    )


# ------------------------------------------------------------------------------ checkpoints
def _target(V, E, Hd, seed):
    g = torch.Generator().manual_seed(seed)
    emb = torch.randn(V, E, generator=g)
    head = torch.randn(V, Hd, generator=g) * 0.1
    target = stub_target(V, E, Hd, torch.float32)
    with torch.no_grad():
        target.model.embed_tokens.weight.copy_(emb)
        target.lm_head.weight.copy_(head)
    return target, emb, head


def gen_checkpoints(ref) -> None:
    """Small SpecForge-style local-head checkpoints of every kind the reference loads,
    the reference's verdict on each (kind, parsed attributes, fused weights, forward
    outputs or the error message) — the pin for the drop-in ``dels.py``."""
    out_dir = HERE / "ckpt"
    out_dir.mkdir(exist_ok=True)
    V, E, G, r, Hd = 64, 8, 16, 4, 12
    target, emb, head = _target(V, E, Hd, 42)
    torch.save({"embed": emb, "lm_head": head}, out_dir / "target.pt")
    g = torch.Generator().manual_seed(7)

    def rnd(*shape, scale=0.3):
        return torch.randn(*shape, generator=g) * scale

    gru = {"prefix_gru.weight_ih_l0": rnd(3 * G, E), "prefix_gru.weight_hh_l0": rnd(3 * G, G)}
    cases = {}
    # (a) direct-vocab RNN head with its own embedding, SiLU rank activation
    cases["direct_vocab"] = {
        "model_config": {"rnn_parameterization": "direct_vocab", "vocab_size": V, "embed_dim": E,
                         "gru_hidden_dim": G, "low_rank_dim": r, "rank_activation": "silu", "shift_label": True},
        "model_state_dict": {**gru, "embed_tokens.weight": rnd(V, E), "rank_proj.weight": rnd(r, G),
                             "low_rank_lm_head.weight": rnd(V, r)},
    }
    # (b) target-factorised head: low-rank head = target lm_head . rank_to_hidden (fused at load)
    cases["target_factorized"] = {
        "model_config": {"local_head_parameterization": "target_factorized", "vocab_size": V, "embed_dim": E,
                         "gru_hidden_dim": G, "low_rank_dim": r, "lm_head_mode": "target_lm_head",
                         "pure_draft_prefix_len": 1},
        "model_state_dict": {**gru, "rank_proj.weight": rnd(r, G), "rank_to_hidden.weight": rnd(Hd, r),
                             "embed_tokens.weight": emb.clone(), "target_lm_head.weight": head.clone()},
    }
    # (c) low-rank head whose weight comes from a separate merged file
    cases["merged_head"] = {
        "model_config": {"vocab_size": V, "embed_dim": E, "gru_hidden_dim": G, "low_rank_dim": r},
        "model_state_dict": {**gru, "rank_proj.weight": rnd(r, G), "rank_to_hidden.weight": rnd(Hd, r)},
    }
    torch.save({"weight": rnd(V, r)}, out_dir / "merged_head_weight.pt")
    # (c') the same with the target-LM-head mode recorded in the config: loads, and the
    # merged weight replaces the factorised head
    cases["merged_head_target"] = {
        "model_config": {"vocab_size": V, "embed_dim": E, "gru_hidden_dim": G, "low_rank_dim": r,
                         "lm_head_mode": "target_lm_head"},
        "model_state_dict": {**gru, "rank_proj.weight": rnd(r, G), "rank_to_hidden.weight": rnd(Hd, r)},
    }
    # (d) errors: an un-merged input projection; an unexpected tensor
    cases["input_projection"] = {
        "model_config": {"vocab_size": V, "embed_dim": E, "gru_hidden_dim": G, "low_rank_dim": r},
        "model_state_dict": {**gru, "embed_down_proj.weight": rnd(E, E)},
    }
    cases["unexpected_tensor"] = {
        "model_config": {"vocab_size": V, "embed_dim": E, "gru_hidden_dim": G, "low_rank_dim": r},
        "model_state_dict": {**gru, "rank_proj.weight": rnd(r, G), "low_rank_lm_head.weight": rnd(V, r),
                             "mystery.weight": rnd(3)},
    }
    # (e) Markov heads, merged and factorised
    cases["markov_merged"] = {"embedding_weight": rnd(V, r), "lm_head_weight": rnd(V, r)}
    cases["markov_factorized"] = {"model_config": {"rank": r},
                                  "model_state_dict": {"down_proj": rnd(E, r), "up_proj": rnd(r, Hd)}}
    # (f) block-prefix position-mix joint head (suffix gates + its own baseline)
    pm_state = {f"local_head_model.{k}": v for k, v in gru.items()}
    pm_state.update({"local_head_model.rank_proj.weight": rnd(r, G), "local_head_model.rank_to_hidden.weight": rnd(Hd, r),
                     "local_head_model.embed_tokens.weight": emb.clone(), "position_gates": rnd(14, 2),
                     "baseline_logits": rnd(1, V), "optimizer_step": torch.tensor(3)})
    cases["position_mix"] = {
        "model_config": {"method": "block_prefix_position_mix_joint", "dflash_shift_label": False,
                         "local_head_config": {"vocab_size": V, "embed_dim": E, "gru_hidden_dim": G,
                                               "low_rank_dim": r, "rank_activation": "identity",
                                               "lm_head_mode": "target_lm_head"}},
        "model_state_dict": pm_state,
    }
    cases["unknown"] = {"something": 1}

    hidden = rnd(1, 3, G, scale=1.0)
    tokens = torch.tensor([[5], [17], [63]])
    prev = torch.tensor([[1], [2], [40]])
    expected = {}
    arrays = {"hidden": hidden.numpy(), "tokens": tokens.numpy(), "prev": prev.numpy()}
    cpu = torch.device("cpu")
    for name, payload in cases.items():
        path = out_dir / f"{name}.pt"
        torch.save(payload, path)
        rec = {}
        try:
            rec["kind"] = ref.dels.detect_local_head_checkpoint_kind(str(path))
        except ValueError as exc:
            rec["kind_error"] = str(exc)
        try:
            if name.startswith("markov"):
                m = ref.dels.MarkovDeLSLocalHead.from_checkpoint(checkpoint_path=str(path), target_model=target,
                                                                 dtype=torch.float32, device=cpu)
                arrays[f"{name}_logits"] = m.logits_from_token(prev).numpy()
                rec.update(vocab_size=m.vocab_size, rank=m.rank)
            elif name == "position_mix":
                m = ref.dels.PositionMixJointHead.from_checkpoint(checkpoint_path=str(path), target_model=target,
                                                                  block_size=16, dtype=torch.float32, device=cpu)
                a, b = m.alpha_beta_schedules()
                rec.update(alpha=a, beta=b, shift_label=m.shift_label, pure=m.pure_draft_prefix_len)
                arrays[f"{name}_baseline"] = m.baseline_logits.numpy()
                arrays[f"{name}_logits"] = m.logits_from_hidden(hidden).numpy()
                arrays[f"{name}_advance"] = m.advance(tokens, hidden).numpy()
            elif name != "unknown":
                kw = ({"merged_lm_head_path": str(out_dir / "merged_head_weight.pt")}
                      if name.startswith("merged_head") else {})
                m = ref.dels.DeLSLocalHead.from_checkpoint(checkpoint_path=str(path), target_model=target,
                                                           dtype=torch.float32, device=cpu, **kw)
                rec.update(lm_head_mode=m.lm_head_mode, pure=m.pure_draft_prefix_len, shift_label=m.shift_label,
                           rank_activation=m.rank_activation)
                arrays[f"{name}_low_rank_lm_head"] = m.low_rank_lm_head.weight.detach().numpy()
                arrays[f"{name}_logits"] = m.logits_from_hidden(hidden).numpy()
                arrays[f"{name}_advance"] = m.advance(tokens, hidden).numpy()
                arrays[f"{name}_empty_hidden"] = m.init_empty_hidden(3, device=cpu).numpy()
        except ValueError as exc:
            rec["load_error"] = str(exc)
        expected[name] = rec
    (out_dir / "expected.json").write_text(json.dumps(expected, indent=1, sort_keys=True) + "\n")
    np.savez_compressed(out_dir / "outputs.npz", **arrays)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout's code/ directory")
    ap.add_argument("--only", nargs="*", default=None,
                    help="generate only these groups (schedules priors scorer runners domino accept checkpoints)")
    ap.add_argument("--domino-fused-worker", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    if args.domino_fused_worker:
        torch.set_num_threads(4)
        domino_fused_worker(args.domino_fused_worker)
        return
    import dels as ref_dels  # noqa: E402
    import dflash as ref_dflash  # noqa: E402
    import kernel.dels as ref_kernel_dels  # noqa: E402
    import kernel.domino as ref_kernel_domino  # noqa: E402
    import kernel.markov_dels as ref_kernel_markov  # noqa: E402

    ref = types.SimpleNamespace(dels=ref_dels, dflash=ref_dflash, kernel_dels=ref_kernel_dels,
                                kernel_markov=ref_kernel_markov, kernel_domino=ref_kernel_domino)
    torch.set_num_threads(4)
    groups = {
        "schedules": lambda: gen_schedules(ref),
        "priors": lambda: gen_priors(ref),
        "scorer": lambda: gen_scorer(ref),
        "runners": lambda: gen_runners(ref),
        "domino": lambda: gen_domino(ref, Path(args.reference)),
        "accept": gen_accept,
        "checkpoints": lambda: gen_checkpoints(ref),
    }
    for name, fn in groups.items():
        if args.only is None or name in args.only:
            fn()
    for p in sorted(HERE.glob("*.npz")) + sorted(HERE.glob("*.json")) + sorted((HERE / "ckpt").glob("*")):
        print(f"{p.name}: {p.stat().st_size} bytes")


if __name__ == "__main__":
    main()
