"""CUDA-graph runner for block-prefix DeLS greedy correction, on the B200 kernels.

Drop-in for ``kernel.dels.DeLSGraphRunner`` of the reference (code/kernel/dels.py:214-478):
same constructor keywords, same ``ValueError`` checks, same ``__call__(prefix_ids,
base_logits) -> LongTensor[B, steps]`` returning a fresh tensor, same static buffers
(``static_prefix_ids``, ``static_base_logits``, ``static_out``), warm-up on a side
stream and capture into ``self.graph``.  At 1-4 rows each captured step is three
``libdels_b200.so`` kernels:

  1. the GRU gates of the previous token (input-table row, gh, h), the token decoded from
     the previous step's packed key (``dels_gru_gates_bf16``);
  2. the rank projection + activation + alpha_step scaling, the step's key slot reset
     (``dels_rank_gemv_bf16``);
  3. the fused scorer on tcgen05 tensor cores: base logits + low-rank logits - beta *
     prior, argmax with the lowest index on ties, as the step's packed key, while two
     helper warps per CTA compute the next step's gh = bf16(W_hh h + b_hh), which needs
     h but not the token (``dels_fused_argmax_base_gru_bf16``);

and one keys decode per call fills the tokens.  With ``DELS_RUNNER_OVERLAP_ROWS`` the
gates of up to that many rows are fused into the rank GEMV instead
(``dels_gru_rank_gemv_bf16``, two kernels per step; measured slower).  At 5-8 rows a step is the GRU step
kernel (``dels_gru_step_bf16``), the rank GEMV and the scorer; from ``DELS_RUNNER_TC_ROWS``
(9) rows up W_hh h and the rank projection run as tensor-core GEMMs
(``dels_gru_step_tc_bf16``, ``dels_rank_project_bf16``).

alpha / beta live in device arrays indexed by step, so one graph serves a schedule;
the reference instead bakes them into the Triton kernels as constexprs (:404-409).
The local head must be bf16 (the reference benchmark always loads it in bf16,
code/benchmark.py:303-309); other dtypes raise ``ValueError``.
"""

from __future__ import annotations

import os

import torch

from dels_b200 import ops


class DeLSGraphRunner:
    """
    CUDA Graph runner for block-prefix DeLS greedy correction.

    Captures the fixed-shape suffix rollout used by the HF benchmark; every step runs
    on hand-written sm_100a kernels (GRU step, rank projection, fused low-rank
    LM-head mix + argmax).
    """

    def __init__(
        self,
        *,
        local_head,
        batch_size: int,
        steps: int,
        vocab_size: int,
        alpha_values: list[float],
        beta_values: list[float],
        baseline_logits: torch.Tensor | None,
        device: torch.device,
    ):
        if steps <= 0:
            raise ValueError(f"DeLSGraphRunner requires steps > 0, got {steps}.")
        if len(alpha_values) != steps or len(beta_values) != steps:
            raise ValueError(
                "DeLS graph alpha/beta schedules must match steps: "
                f"steps={steps}, alpha={len(alpha_values)}, beta={len(beta_values)}."
            )
        if any(float(beta) != 0.0 for beta in beta_values) and baseline_logits is None:
            raise ValueError("DeLS graph requires baseline_logits when any beta is nonzero.")

        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("DeLSGraphRunner runs on a CUDA device (sm_100a kernels only).")
        self.local_head = local_head
        self.batch_size = int(batch_size)
        self.steps = int(steps)
        self.vocab_size = int(vocab_size)
        self.alpha_values = [float(x) for x in alpha_values]
        self.beta_values = [float(x) for x in beta_values]

        dtype = local_head.rank_proj.weight.dtype
        if dtype != torch.bfloat16:
            raise ValueError(f"DeLSGraphRunner kernels are bf16; the local head is {dtype}.")
        self.rank_dim = int(local_head.low_rank_lm_head.weight.shape[1])
        self._r = ops.round8(self.rank_dim)  # carried rank width, zero-padded to a multiple of 8
        # Kept for the reference's log line (code/benchmark.py:481-484): the fused path
        # is always used here.
        self._can_triton_fuse = True
        activation = getattr(local_head, "rank_activation", "identity")
        if activation not in ops.ACTIVATIONS:
            raise ValueError(f"Unsupported DeLS rank_activation={activation!r}.")
        self._activation = activation

        gru = local_head.prefix_gru
        if gru.num_layers != 1 or gru.bidirectional:
            raise ValueError("DeLS graph runner supports only a single unidirectional GRU.")
        self.gru_hidden_dim = int(gru.hidden_size)
        with torch.no_grad():
            self.gru_w_ih = gru.weight_ih_l0.detach().to(device).contiguous()
            self.gru_w_hh = gru.weight_hh_l0.detach().to(device).contiguous()
            self.gru_b_ih = gru.bias_ih_l0.detach().to(device).contiguous() if gru.bias else None
            self.gru_b_hh = gru.bias_hh_l0.detach().to(device).contiguous() if gru.bias else None

            # gi table = F.linear(embed, W_ih, b_ih) (code/kernel/dels.py:265-268) on the
            # tensor-core projection kernel: one bf16 rounding of an fp32 accumulation.  The
            # embedding width is zero-padded to a multiple of 8 for the TMA tiles.
            E8 = ops.round8(self.gru_w_ih.shape[1])
            embed_weight = ops.zero_pad(local_head.embed_tokens.weight.detach().to(device).contiguous(), cols=E8)
            self._gru_input_proj_table = ops.linear_bf16(embed_weight, ops.zero_pad(self.gru_w_ih, cols=E8),
                                                         self.gru_b_ih)

            self.rank_weight = ops.zero_pad(local_head.rank_proj.weight.detach().to(device).contiguous(),
                                            rows=self._r)
            self.rank_bias = (
                ops.zero_pad(local_head.rank_proj.bias.detach().to(device).contiguous(), rows=self._r)
                if local_head.rank_proj.bias is not None
                else None
            )
            self.lm_head_weight = ops.zero_pad(local_head.low_rank_lm_head.weight.detach().to(device).contiguous(),
                                               cols=self._r)

            baseline_flat = torch.zeros(self.vocab_size, dtype=dtype, device=device)
            if baseline_logits is not None:
                baseline_numel = int(baseline_logits.numel())
                if baseline_numel != self.vocab_size:
                    raise ValueError(
                        "DeLS graph baseline vocab size mismatch: "
                        f"baseline={baseline_numel}, vocab={self.vocab_size}."
                    )
                baseline_flat.copy_(baseline_logits.to(device=device, dtype=dtype).reshape(-1))
        self.baseline_logits = baseline_flat.contiguous()
        self.has_baseline = baseline_logits is not None
        # the scorer reads the prior in fp32 (exactly the bf16 values above)
        self._prior_f32 = self.baseline_logits.to(torch.float32) if self.has_baseline else None

        B, G, r, S = self.batch_size, self.gru_hidden_dim, self._r, self.steps
        self.static_prefix_ids = torch.zeros(B, 1, dtype=torch.long, device=device)
        self._alloc_step_inputs(dtype, device)
        self.static_out = torch.zeros(B, S, dtype=torch.long, device=device)

        self._alpha = torch.tensor(self.alpha_values, dtype=torch.float32, device=device)
        # beta == 0 at a step skips the prior like the reference (:382); a zero beta
        # contributes nothing, so the device array simply holds the schedule.
        self._beta = torch.tensor(self.beta_values, dtype=torch.float32, device=device)
        self._tokens = torch.zeros(S, B, dtype=torch.long, device=device)  # step-major token slots
        self._h = [torch.zeros(B, G, dtype=dtype, device=device) for _ in range(2)]
        self._s_scaled = torch.zeros(B, r, dtype=dtype, device=device)
        self._keys = torch.empty(B, dtype=torch.int64, device=device)
        self._ws = ops.Workspace(1 << 12, device)
        self._outs = [ops.ScoreOut(tokens=self._tokens[i], scores=None, keys=self._keys) for i in range(S)]
        # From DELS_RUNNER_TC_ROWS rows up (default 9) the GRU's W_hh product and the rank
        # projection run as tensor-core split-K GEMMs (then the gates / the rank
        # finalisation); below it one warp per weight row does each in a single launch.
        tc_rows = int(os.environ.get("DELS_RUNNER_TC_ROWS", "9"))
        self._tc = B >= tc_rows and self.rank_bias is None
        # Up to DELS_RUNNER_OVERLAP_ROWS rows (default 0: off; at most 4) a step is two
        # kernels: the GRU gates fused into the rank projection (dels_gru_rank_gemv_bf16),
        # then the scorer, whose two helper warps per CTA compute the next step's W_hh h
        # (which needs h but not the token) while the others score
        # (dels_fused_argmax_base_gru_bf16).  Measured slower than the split schedule below
        # once that one was keys-only.
        self._overlap = (B <= min(4, int(os.environ.get("DELS_RUNNER_OVERLAP_ROWS", "0"))) and not self._tc
                         and self._scorer_computes_next_gh())
        # Batches of at most DELS_RUNNER_SPLIT_ROWS rows (default 4, at most 8;
        # DELS_RUNNER_SPLIT_GRU=0 turns it off): the scorer's helper warps compute the next
        # W_hh h, and the step's GRU update shrinks to the gates (dels_gru_gates_bf16)
        # before the rank GEMV, three kernels.  From 5 rows the helpers' work, which grows
        # with the rows, outlasts this runner's scorer (Vr, 78 MB per step).
        self._split_gru = (not self._tc and not self._overlap
                           and B <= min(8, int(os.environ.get("DELS_RUNNER_SPLIT_ROWS", "4")))
                           and os.environ.get("DELS_RUNNER_SPLIT_GRU", "1") != "0"
                           and self._scorer_computes_next_gh())
        if self._tc:
            # the GRU's split-K finalisation evaluates the gates itself (dels_gru_step_tc_bf16;
            # DELS_RUNNER_GRU_TC_FUSED=0 runs dels_linear_bf16 then dels_gru_gates_bf16)
            self._gru_tc_fused = os.environ.get("DELS_RUNNER_GRU_TC_FUSED", "1") != "0"
            need = max(ops.linear_workspace_bytes(B, G, 3 * G), ops.rank_workspace_bytes(B, G, r),
                       int(ops._lib.query("dels_gru_step_tc_workspace_bytes", B, G)))
            self._tc_ws = ops.Workspace(need, device)
        # The split schedule reads the previous step's packed keys in its gates kernel too
        # (DELS_RUNNER_SPLIT_KEYS=0: each scorer decodes its own tokens).
        self._split_keys = self._split_gru and os.environ.get("DELS_RUNNER_SPLIT_KEYS", "1") != "0"
        # From 5 rows (GRU step kernel or tensor-core GRU, rank projection, scorer), and in
        # DeLSFusedGraphRunner at every batch, the GRU reads the previous step's packed keys
        # as well (DELS_RUNNER_PLAIN_KEYS=0: each scorer decodes its own tokens)
        self._plain_keys = (not self._overlap and not self._split_gru
                            and os.environ.get("DELS_RUNNER_PLAIN_KEYS", "1") != "0")
        self._keys_only = self._overlap or self._split_keys or self._plain_keys
        if self._keys_only:
            # Per-step packed argmax keys: each step's scorer only writes keys (no in-kernel
            # decode: no last-CTA count, fence or decode at the end of every step), the next
            # step's GRU gates (fused into the rank GEMV, or their own kernel) decode the
            # token they need, and one decode per call fills the token slots.
            self._step_keys = torch.empty(S, B, dtype=torch.int64, device=device)
            self._key_outs = [ops.ScoreOut(tokens=None, scores=None, keys=self._step_keys[i]) for i in range(S)]
        if self._tc or self._overlap or self._split_gru:
            self._gh = torch.empty(B, 3 * G, dtype=dtype, device=device)
            # the first step's h is zero, so its gh is the bias alone
            self._gh0 = torch.zeros(B, 3 * G, dtype=dtype, device=device)
            if self.gru_b_hh is not None:
                self._gh0.copy_(self.gru_b_hh.to(dtype)[None, :].expand(B, -1))

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
        if h_in is None:
            return ops.gru_gates(tokens, self._gru_input_proj_table, self._gh0, h_in, h_out, ws=self._ws,
                                 tokens_are_keys=keys)
        if self._gru_tc_fused:
            # W_hh h as a split-K GEMM whose finalisation evaluates the gates (one kernel less)
            return ops.gru_step_tc(tokens, self._gru_input_proj_table, self.gru_w_hh, h_in, h_out,
                                   b_hh=self.gru_b_hh, ws=self._tc_ws, tokens_are_keys=keys)
        gh = ops.linear_bf16(h_in, self.gru_w_hh, self.gru_b_hh, out=self._gh, ws=self._tc_ws)
        return ops.gru_gates(tokens, self._gru_input_proj_table, gh, h_in, h_out, ws=self._ws, tokens_are_keys=keys)

    def _rank(self, h_cur, step: int, keys=None):
        keys = self._keys if keys is None else keys
        if not self._tc:
            ops.rank_gemv(h_cur, self.rank_weight, self._alpha[step : step + 1], self._s_scaled,
                          bias=self.rank_bias, activation=self._activation, keys=keys, ws=self._ws)
        else:
            ops.rank_project_bf16(h_cur, self.rank_weight, self._alpha[step : step + 1], n_pos=1,
                                  activation=self._activation, s_scaled=self._s_scaled, keys=keys,
                                  want_state=False, ws=self._tc_ws)

    def _forward_gh_on_scorer(self):
        tokens, h_prev, gh, cur = self.static_prefix_ids[:, 0], None, self._gh0, 0
        for step in range(self.steps):
            h_new = self._h[cur]
            if self._overlap:
                ops.gru_rank_gemv(tokens, self._gru_input_proj_table, gh, h_prev, h_new, self.rank_weight,
                                  self._alpha[step : step + 1], self._s_scaled, bias=self.rank_bias,
                                  activation=self._activation, keys=self._step_keys[step], ws=self._ws,
                                  tokens_are_keys=step > 0)
            else:
                ops.gru_gates(tokens, self._gru_input_proj_table, gh, h_prev, h_new, ws=self._ws,
                              tokens_are_keys=self._split_keys and step > 0)
                self._rank(h_new, step, keys=self._step_keys[step] if self._split_keys else None)
            if step + 1 < self.steps:
                # the scorer's helper warps compute the next step's gh = bf16(W_hh h_new + b_hh)
                self._score(step, next_gh=(h_new, self._gh))
            else:
                self._score(step)
            if self._keys_only:
                tokens = self._step_keys[step]
            else:
                tokens = self._tokens[step]
            h_prev, gh, cur = h_new, self._gh, cur ^ 1
        if self._keys_only:
            ops.keys_decode(self._step_keys.view(-1), tokens=self._tokens.view(-1), with_scores=False)
        self.static_out.copy_(self._tokens.t())

    def _forward_impl(self):
        if self._overlap or self._split_gru:
            return self._forward_gh_on_scorer()
        prefix = self.static_prefix_ids[:, 0]
        h_cur = self._gru(prefix, None, self._h[0])
        nxt = 1
        keys = self._plain_keys
        for step in range(self.steps):
            self._rank(h_cur, step, keys=self._step_keys[step] if keys else None)
            self._score(step)
            if step + 1 < self.steps:
                prev = self._step_keys[step] if keys else self._tokens[step]
                h_cur = self._gru(prev, h_cur, self._h[nxt], keys=keys)
                nxt ^= 1
        if keys:
            ops.keys_decode(self._step_keys.view(-1), tokens=self._tokens.view(-1), with_scores=False)
        self.static_out.copy_(self._tokens.t())

    # -- the per-step inputs and scorer; DeLSFusedGraphRunner overrides these ----------
    def _alloc_step_inputs(self, dtype, device):
        self.static_base_logits = torch.zeros(self.batch_size, self.steps, self.vocab_size, dtype=dtype,
                                              device=device)

    def _scorer_computes_next_gh(self) -> bool:
        return True

    def _score(self, step: int, next_gh=None):
        out = self._key_outs[step] if self._keys_only else self._outs[step]
        if next_gh is not None:
            h, gh_out = next_gh
            ops.fused_argmax_base_gru_bf16(
                self.static_base_logits[:, step, :], self._s_scaled, self.lm_head_weight, self._prior_f32,
                self._beta[step : step + 1], self.gru_w_hh, self.gru_b_hh, h, gh_out, keys_ready=True,
                out=out, ws=self._ws,
            )
            return
        ops.fused_argmax_base_bf16(
            self.static_base_logits[:, step, :], self._s_scaled, self.lm_head_weight,
            self._prior_f32, self._beta[step : step + 1], n_pos=1, keys_ready=True, out=out, ws=self._ws,
        )

    @torch.inference_mode()
    def __call__(
        self,
        prefix_ids: torch.Tensor,
        base_logits: torch.Tensor,
    ) -> torch.Tensor:
        self.static_prefix_ids.copy_(prefix_ids)
        self.static_base_logits.copy_(base_logits)
        self.graph.replay()
        return self.static_out.clone()


class DeLSFusedGraphRunner(DeLSGraphRunner):
    """DeLS rollout that takes the DFlash draft hidden states instead of the long logits.

    The reference materialises ``base_logits = target.lm_head(parallel_hiddens)``
    ([B, 15, V], code/dflash.py:468), slices positions 1..steps into a contiguous copy and
    copies that into the runner (:482-485).  Here the runner owns the LM head and takes
    ``__call__(prefix_ids [B, 1], parallel_hiddens [B, steps, H])`` (the hidden states of
    the positions the reference feeds as base logits).  Two schedules, picked by batch:

    * ``B >= DELS_FUSED_RUNNER_ROWS`` (default 192): every step scores
          h_t . W_lm + alpha_t * act(W_rank g_t) . Vr - beta_t * prior
      inside the tensor-core scorer (``dels_fused_argmax_bf16``), so the long logits are
      never written.  A step streams the LM head once; with a few hundred rows per step the
      scorer is tensor-bound, the FLOPs equal those of one big GEMM over all positions,
      and the [B, steps, V] round trip disappears.
    * smaller batches: the rollout's steps depend on each other, so a per-step scorer
      would stream the whole LM head ``steps`` times for a handful of rows.  Instead the
      graph starts with one GEMM over all B x steps hidden rows (``dels_linear_bf16``,
      which writes bf16 logits straight from its epilogue into the runner's own buffer:
      one pass over W, no slice copy, no copy-in), then runs the base-logit rollout.
      Base logits are bf16-rounded here, as in the reference.
    """

    def __init__(self, *, target_lm_head_weight: torch.Tensor, **kwargs):
        w = target_lm_head_weight.detach()
        if w.dim() != 2 or int(w.shape[0]) != int(kwargs["vocab_size"]):
            raise ValueError(
                f"target LM head weight {tuple(w.shape)} does not match vocab_size={kwargs['vocab_size']}."
            )
        self._lm_weight = w.to(device=kwargs["device"], dtype=torch.bfloat16).contiguous()
        self.hidden_size = int(w.shape[1])
        self._fused = int(kwargs["batch_size"]) >= int(os.environ.get("DELS_FUSED_RUNNER_ROWS", "192"))
        super().__init__(**kwargs)

    def _alloc_step_inputs(self, dtype, device):
        B, S = self.batch_size, self.steps
        self.static_parallel_hiddens = torch.zeros(B, S, self.hidden_size, dtype=dtype, device=device)
        if not self._fused:
            self.static_base_logits = torch.zeros(B, S, self.vocab_size, dtype=dtype, device=device)
            self._lm_ws = ops.Workspace(ops.linear_workspace_bytes(B * S, self.hidden_size, self.vocab_size),
                                        device)

    def _forward_impl(self):
        if not self._fused:
            B, S = self.batch_size, self.steps
            ops.linear_bf16(self.static_parallel_hiddens.view(B * S, self.hidden_size), self._lm_weight,
                            out=self.static_base_logits.view(B * S, self.vocab_size), ws=self._lm_ws)
        super()._forward_impl()

    def _scorer_computes_next_gh(self) -> bool:
        return not self._fused  # the hidden-state scorer has no helper warps

    def _score(self, step: int, next_gh=None):
        if not self._fused:
            return super()._score(step, next_gh)
        if next_gh is not None:
            raise RuntimeError("the per-step fused scorer does not compute the GRU projection")
        ops.fused_argmax_bf16(
            self.static_parallel_hiddens[:, step, :], self._lm_weight, self._s_scaled, self.lm_head_weight,
            self._prior_f32, self._beta[step : step + 1], n_pos=1, keys_ready=True,
            out=self._key_outs[step] if self._keys_only else self._outs[step], ws=self._ws,
        )

    @torch.inference_mode()
    def __call__(self, prefix_ids: torch.Tensor, parallel_hiddens: torch.Tensor) -> torch.Tensor:
        self.static_prefix_ids.copy_(prefix_ids)
        self.static_parallel_hiddens.copy_(parallel_hiddens)
        self.graph.replay()
        return self.static_out.clone()
