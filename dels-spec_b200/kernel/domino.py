"""CUDA-graph runner for the Domino draft correction, on the B200 kernels.

Drop-in for ``kernel.domino.DraftCorrectionGraphRunner`` of the reference
(code/kernel/domino.py:232-520): same constructor keywords and checks, same
``__call__(prefix_ids, parallel_hiddens, base_logits, guidance_alpha=None) ->
LongTensor[B, steps]`` returning a fresh tensor, same static buffers
(``static_prefix_ids``, ``static_parallel_hiddens``, ``static_base_logits``,
``static_out``), warm-up on a side stream and capture into ``self.graph``.

Per call (all on ``libdels_b200.so``):

  z = F.linear(parallel_hiddens, W_z, b1)          ``dels_linear_bf16`` (tcgen05, once)
  h = GRU over the prefix tokens from zero           ``dels_gru_step_bf16`` per token
  per step t:
    s' = bf16(alpha * SiLU(z_t + W_s h))             ``dels_correction_mid_bf16``
    tok = argmax(s' . fc2^T + alpha * b2 + base_t)   ``dels_fused_argmax_base_bf16``
                                                     (prior = b2, beta = -alpha)
    h = GRUCell(table[tok], h)                       ``dels_gru_step_bf16``

At 1-8 rows W_hh h of the GRU update moves onto two helper warps per CTA of the scorer
(``dels_fused_argmax_base_gru_bf16``: it needs h but not the token) and only the gates
stay between steps, as their own kernel decoding the previous step's packed key
(``dels_gru_gates_bf16``; with ``DELS_RUNNER_OVERLAP_ROWS`` fused into the next step's
correction layer, ``dels_gru_correction_mid_bf16``, measured slower).
From ``DELS_RUNNER_TC_ROWS`` (9) rows up W_hh h and W_s h run on the tensor-core GEMMs
(``dels_gru_step_tc_bf16``, ``dels_correction_mid_tc_bf16``).

The correction MLP must be Linear -> SiLU -> Linear (the released Domino head,
code/dflash.py:271-276, and the only form the reference fuses, :283-291); its weights
must be bf16.  Other forms raise ``ValueError``.
"""

from __future__ import annotations

import os

from typing import Tuple

import torch
import torch.nn as nn

from dels_b200 import ops


def unwrap_correction_mlp(embed_proj: nn.Module) -> Tuple[nn.Linear, nn.Module, nn.Linear]:
    """(fc1, middle, fc2) of ``nn.Sequential(Linear(H + G, M), ..., Linear(M, V))``; the
    input of fc1 is concat([z, s]) (code/kernel/domino.py:15-50, same errors)."""
    if not isinstance(embed_proj, nn.Sequential):
        raise TypeError("Graph runner requires draft_model.embed_proj to be nn.Sequential.")
    layers = list(embed_proj.children())
    if len(layers) < 2:
        raise ValueError("embed_proj must contain at least two layers.")
    if not isinstance(layers[0], nn.Linear):
        raise ValueError("embed_proj first layer must be nn.Linear.")
    if not isinstance(layers[-1], nn.Linear):
        raise ValueError("embed_proj last layer must be nn.Linear.")
    middle = nn.Sequential(*layers[1:-1]) if len(layers) > 2 else nn.Identity()
    return layers[0], middle, layers[-1]


def _is_silu(middle: nn.Module) -> bool:
    if isinstance(middle, nn.SiLU):
        return True
    inner = list(middle.children()) if isinstance(middle, nn.Sequential) else []
    return len(inner) == 1 and isinstance(inner[0], nn.SiLU)


def _bf16(t: torch.Tensor | None, device: torch.device) -> torch.Tensor | None:
    return None if t is None else t.detach().to(device=device, dtype=torch.bfloat16).contiguous()


class DraftCorrectionGraphRunner:
    """
    CUDA Graph runner for block draft correction (greedy), every step on hand-written
    sm_100a kernels: correction-MLP hidden layer, fused fc2 GEMV + bias + base logits +
    argmax on tcgen05 tensor cores, and the GRU cell over the realised token.
    """

    def __init__(
        self,
        draft_model: nn.Module,
        target_model: nn.Module,
        batch_size: int,
        steps: int,
        hidden_dim: int,
        gru_hidden_dim: int,
        vocab_size: int,
        prefix_token_count: int,
        device: torch.device,
        guidance_alpha: float = 1.0,
    ):
        self.steps = int(steps)
        self.draft_model = draft_model
        self.target_model = target_model
        self.prefix_token_count = int(prefix_token_count)
        self.gru_hidden_dim = int(gru_hidden_dim)
        self.guidance_alpha = float(guidance_alpha)
        self.batch_size = int(batch_size)
        self.vocab_size = int(vocab_size)

        fc1, self.middle, fc2 = unwrap_correction_mlp(draft_model.embed_proj)
        expected_in = hidden_dim + gru_hidden_dim
        if fc1.in_features != expected_in:
            raise ValueError(
                f"Correction MLP input dim mismatch: got {fc1.in_features}, "
                f"expected {expected_in} = hidden_dim + gru_hidden_dim."
            )
        self._middle_is_silu = _is_silu(self.middle)
        if not self._middle_is_silu:
            raise ValueError("DraftCorrectionGraphRunner (sm_100a kernels) needs a SiLU correction MLP "
                             f"(Linear -> SiLU -> Linear); got middle={self.middle!r}.")
        # Kept for the reference's log line: the fused path is always taken here.
        self._can_triton_fuse = True

        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("DraftCorrectionGraphRunner runs on a CUDA device (sm_100a kernels only).")
        dtype = next(draft_model.parameters()).dtype
        if dtype != torch.bfloat16:
            raise ValueError(f"DraftCorrectionGraphRunner kernels are bf16; the draft model is {dtype}.")
        if self.prefix_token_count < 1:
            raise ValueError(f"prefix_token_count must be >= 1, got {prefix_token_count}.")

        gru = draft_model.prefix_gru
        assert gru.num_layers == 1 and not gru.bidirectional
        B, S, H, G = self.batch_size, self.steps, int(hidden_dim), self.gru_hidden_dim
        self.hidden_dim = H
        self.mlp_hidden_dim = int(fc1.out_features)
        M = ops.round8(self.mlp_hidden_dim)  # carried width, zero-padded to a multiple of 8
        self._m = M
        with torch.no_grad():
            w1 = fc1.weight.detach()
            self.w_z = ops.zero_pad(_bf16(w1[:, :H], device), rows=M)
            self.w_s = ops.zero_pad(_bf16(w1[:, H:], device), rows=M)
            self.fc1_bias = ops.zero_pad(_bf16(fc1.bias, device), rows=M)
            self.fc2_weight = ops.zero_pad(_bf16(fc2.weight, device), cols=M)
            self.fc2_bias = _bf16(fc2.bias, device)
            self.gru_w_ih = _bf16(gru.weight_ih_l0, device)
            self.gru_w_hh = _bf16(gru.weight_hh_l0, device)
            self.gru_b_ih = _bf16(gru.bias_ih_l0, device) if gru.bias else None
            self.gru_b_hh = _bf16(gru.bias_hh_l0, device) if gru.bias else None
            # gi table = F.linear(embed, W_ih, b_ih) (code/kernel/domino.py:323-327); the
            # embedding width is zero-padded to a multiple of 8 for the TMA tiles.
            E8 = ops.round8(self.gru_w_ih.shape[1])
            embed_weight = ops.zero_pad(_bf16(target_model.model.embed_tokens.weight, device), cols=E8)
            self._gru_input_proj_table = ops.linear_bf16(embed_weight, ops.zero_pad(self.gru_w_ih, cols=E8),
                                                         self.gru_b_ih)
        if int(self.fc2_weight.shape[0]) != self.vocab_size:
            raise ValueError(f"fc2 has {self.fc2_weight.shape[0]} outputs, vocab_size is {self.vocab_size}.")

        self.static_prefix_ids = torch.zeros(B, self.prefix_token_count, dtype=torch.long, device=device)
        self.static_parallel_hiddens = torch.zeros(B, S, H, dtype=dtype, device=device)
        self.static_base_logits = torch.zeros(B, S, self.vocab_size, dtype=dtype, device=device)
        self.static_out = torch.zeros(B, S, dtype=torch.long, device=device)

        # alpha * b2 enters the scorer as -beta * prior with prior = b2, beta = -alpha
        self._alpha = torch.tensor([self.guidance_alpha], dtype=torch.float32, device=device)
        self._beta = torch.tensor([-self.guidance_alpha], dtype=torch.float32, device=device)
        self._prior_f32 = self.fc2_bias.to(torch.float32).contiguous() if self.fc2_bias is not None else None
        self._z = torch.zeros(B * S, M, dtype=dtype, device=device)
        self._h = [torch.zeros(B, G, dtype=dtype, device=device) for _ in range(2)]
        self._s_scaled = torch.zeros(B, M, dtype=dtype, device=device)
        self._tokens = torch.zeros(max(S, 1), B, dtype=torch.long, device=device)  # step-major
        self._keys = torch.empty(B, dtype=torch.int64, device=device)
        self._ws = ops.Workspace(1 << 12, device)
        self._ws_lin = ops.Workspace(1 << 12, device)
        self._outs = [ops.ScoreOut(tokens=self._tokens[i], scores=None, keys=self._keys) for i in range(S)]
        # From DELS_RUNNER_TC_ROWS rows up (default 9) the GRU's W_hh product and the
        # correction MLP's W_s product run as tensor-core split-K GEMMs, then the gates /
        # the SiLU epilogue (as in kernel/dels.py).
        self._tc = B >= int(os.environ.get("DELS_RUNNER_TC_ROWS", "9"))
        if self._tc:
            # the GRU's split-K finalisation evaluates the gates itself (dels_gru_step_tc_bf16;
            # DELS_RUNNER_GRU_TC_FUSED=0 runs dels_linear_bf16 then dels_gru_gates_bf16)
            self._gru_tc_fused = os.environ.get("DELS_RUNNER_GRU_TC_FUSED", "1") != "0"
            self._tc_ws = ops.Workspace(max(ops.linear_workspace_bytes(B, G, 3 * G),
                                            ops.correction_mid_tc_workspace_bytes(B, G, M),
                                            int(ops._lib.query("dels_gru_step_tc_workspace_bytes", B, G))), device)
            self._gh0 = torch.zeros(B, 3 * G, dtype=dtype, device=device)
            if self.gru_b_hh is not None:
                self._gh0.copy_(self.gru_b_hh[None, :].expand(B, -1))
        # Up to DELS_RUNNER_OVERLAP_ROWS rows (default 0: off; at most 4) a step
        # after the first is two kernels: the previous token's GRU gates fused into the
        # correction layer (dels_gru_correction_mid_bf16), then the scorer, whose helper
        # warps compute the next update's W_hh h (dels_fused_argmax_base_gru_bf16).
        self._overlap = B <= min(4, int(os.environ.get("DELS_RUNNER_OVERLAP_ROWS", "0"))) and not self._tc
        # Batches of at most DELS_RUNNER_SPLIT_ROWS rows (default 8, at most 8;
        # DELS_RUNNER_SPLIT_GRU=0 turns it off): the same helper warps, with the GRU update
        # reduced to its gates (dels_gru_gates_bf16).  This scorer streams fc2 (311 MB per
        # step), long enough to hide the helpers' W_hh h at 5-8 rows too.
        self._split_gru = (not self._tc and not self._overlap
                           and B <= min(8, int(os.environ.get("DELS_RUNNER_SPLIT_ROWS", "8")))
                           and os.environ.get("DELS_RUNNER_SPLIT_GRU", "1") != "0")
        if self._tc or self._overlap or self._split_gru:
            self._gh = torch.empty(B, 3 * G, dtype=dtype, device=device)
        # the split schedule reads the previous step's packed keys in its gates kernel too
        # (DELS_RUNNER_SPLIT_KEYS=0: each scorer decodes its own tokens)
        self._split_keys = self._split_gru and os.environ.get("DELS_RUNNER_SPLIT_KEYS", "1") != "0"
        # outside the split schedule the GRU update between steps reads the previous step's
        # packed keys as well (DELS_RUNNER_PLAIN_KEYS=0: each scorer decodes its own tokens)
        self._plain_keys = (not self._overlap and not self._split_gru
                            and os.environ.get("DELS_RUNNER_PLAIN_KEYS", "1") != "0")
        self._keys_only = self._overlap or self._split_keys or self._plain_keys
        if self._keys_only:
            # per-step packed argmax keys: keys-only scorer calls, the next step's gates (fused
            # or their own kernel) decode the token they need, one decode per call fills the
            # token slots
            self._step_keys = torch.empty(max(S, 1), B, dtype=torch.int64, device=device)
            self._key_outs = [ops.ScoreOut(tokens=None, scores=None, keys=self._step_keys[i]) for i in range(S)]

        ops.init(device)
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.inference_mode(), torch.cuda.stream(stream):
            for _ in range(3):
                self._forward_impl()
        torch.cuda.current_stream(device).wait_stream(stream)

        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(self.graph):
            self._forward_impl()

    def _gru(self, tokens, h_in, h_out, keys: bool = False):
        # keys: `tokens` holds the previous step's packed argmax keys
        if not self._tc:
            return ops.gru_step(tokens, self._gru_input_proj_table, self.gru_w_hh, h_in, h_out, b_hh=self.gru_b_hh,
                                ws=self._ws, tokens_are_keys=keys)
        if h_in is not None and self._gru_tc_fused:
            # W_hh h as a split-K GEMM whose finalisation evaluates the gates (one kernel less)
            return ops.gru_step_tc(tokens, self._gru_input_proj_table, self.gru_w_hh, h_in, h_out,
                                   b_hh=self.gru_b_hh, ws=self._tc_ws, tokens_are_keys=keys)
        gh = self._gh0 if h_in is None else ops.linear_bf16(h_in, self.gru_w_hh, self.gru_b_hh, out=self._gh,
                                                           ws=self._tc_ws)
        return ops.gru_gates(tokens, self._gru_input_proj_table, gh, h_in, h_out, ws=self._ws, tokens_are_keys=keys)

    def _forward_impl(self):
        B, S, H, M = self.batch_size, self.steps, self.hidden_dim, self._m
        if S > 0:
            ops.linear_bf16(self.static_parallel_hiddens.view(B * S, H), self.w_z, self.fc1_bias, out=self._z,
                            ws=self._ws_lin)
        z = self._z.view(B, S, M)
        h = None
        cur = 0
        for p in range(self.prefix_token_count):
            h = self._gru(self.static_prefix_ids[:, p], h, self._h[cur])
            cur ^= 1
        gh_on_scorer = self._overlap or self._split_gru
        for t in range(S):
            last = t + 1 == S
            keys = self._step_keys[t] if self._keys_only else self._keys
            out = self._key_outs[t] if self._keys_only else self._outs[t]
            if self._overlap and t > 0:
                # the previous token's GRU gates fused into this step's correction layer; the
                # token comes from the previous step's packed key
                h_prev, h = h, self._h[cur]
                cur ^= 1
                ops.gru_correction_mid(self._step_keys[t - 1], self._gru_input_proj_table, self._gh, h_prev, h,
                                       self.w_s, z[:, t, :], self._alpha, self._s_scaled, keys=keys, ws=self._ws,
                                       tokens_are_keys=True)
            elif self._split_gru and t > 0:
                h_prev, h = h, self._h[cur]
                cur ^= 1
                prev = self._step_keys[t - 1] if self._split_keys else self._tokens[t - 1]
                ops.gru_gates(prev, self._gru_input_proj_table, self._gh, h_prev, h, ws=self._ws,
                              tokens_are_keys=self._split_keys)
                ops.correction_mid(h, self.w_s, z[:, t, :], self._alpha, self._s_scaled, keys=keys, ws=self._ws)
            elif self._tc:
                ops.correction_mid_tc(h, self.w_s, z[:, t, :], self._alpha, self._s_scaled, keys=keys,
                                      ws=self._tc_ws)
            else:
                ops.correction_mid(h, self.w_s, z[:, t, :], self._alpha, self._s_scaled, keys=keys, ws=self._ws)
            base_t = self.static_base_logits[:, t, :]
            if gh_on_scorer and not last:
                # the scorer's helper warps compute the next update's gh = bf16(W_hh h + b_hh)
                ops.fused_argmax_base_gru_bf16(base_t, self._s_scaled, self.fc2_weight, self._prior_f32,
                                               self._beta, self.gru_w_hh, self.gru_b_hh, h, self._gh,
                                               keys_ready=True, out=out, ws=self._ws)
            else:
                ops.fused_argmax_base_bf16(base_t, self._s_scaled, self.fc2_weight, self._prior_f32, self._beta,
                                           n_pos=1, keys_ready=True, out=out, ws=self._ws)
            if not last and not gh_on_scorer:
                prev = self._step_keys[t] if self._plain_keys else self._tokens[t]
                h = self._gru(prev, h, self._h[cur], keys=self._plain_keys)
                cur ^= 1
        if S > 0:
            if self._keys_only:
                ops.keys_decode(self._step_keys[:S].reshape(-1), tokens=self._tokens[:S].view(-1), with_scores=False)
            self.static_out.copy_(self._tokens[:S].t())

    @torch.inference_mode()
    def __call__(
        self,
        prefix_ids: torch.Tensor,
        parallel_hiddens: torch.Tensor,
        base_logits: torch.Tensor,
        guidance_alpha: float | None = None,
    ) -> torch.Tensor:
        if guidance_alpha is not None and float(guidance_alpha) != self.guidance_alpha:
            raise ValueError(
                "DraftCorrectionGraphRunner captures a fixed domino guidance alpha; "
                f"got {float(guidance_alpha)} but runner was built with {self.guidance_alpha}."
            )
        self.static_prefix_ids.copy_(prefix_ids)
        self.static_parallel_hiddens.copy_(parallel_hiddens)
        self.static_base_logits.copy_(base_logits)
        self.graph.replay()
        return self.static_out.clone()
