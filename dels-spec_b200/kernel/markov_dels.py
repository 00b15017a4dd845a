"""CUDA-graph runner for greedy Markov DeLS suffix rollout, on the B200 kernels.

Drop-in for ``kernel.markov_dels.MarkovDeLSGraphRunner`` of the reference
(code/kernel/markov_dels.py:139-312): same constructor keywords and ``ValueError``
checks, ``__call__(prev_token_ids, base_logits) -> LongTensor[B, steps]``.  Each
captured step is two kernels: the embedding-row gather of the previous token scaled by
alpha_step (``dels_gather_scaled_rows_bf16``) and the fused tcgen05 scorer over
base + low-rank - beta * prior (``dels_fused_argmax_base_bf16``).  The scorer of each
step writes only its packed (score, index) keys; the next step's gather decodes the
previous key itself, and one ``dels_keys_decode`` per call turns every step's keys into
the output tokens, so no scorer ends with a completion count and a decode of its own.
"""

from __future__ import annotations

import torch

from dels_b200 import ops


class MarkovDeLSGraphRunner:
    """CUDA Graph runner for greedy Markov DeLS suffix rollout."""

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
            raise ValueError(f"MarkovDeLSGraphRunner requires steps > 0, got {steps}.")
        if len(alpha_values) != steps or len(beta_values) != steps:
            raise ValueError(
                "Markov DeLS graph alpha/beta schedules must match steps: "
                f"steps={steps}, alpha={len(alpha_values)}, beta={len(beta_values)}."
            )
        if int(local_head.vocab_size) != int(vocab_size):
            raise ValueError(
                "Markov DeLS local-head vocab size mismatch: "
                f"local_head={local_head.vocab_size}, vocab={vocab_size}."
            )
        if any(float(beta) != 0.0 for beta in beta_values) and baseline_logits is None:
            raise ValueError("Markov DeLS graph requires baseline_logits when any beta is nonzero.")

        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("MarkovDeLSGraphRunner runs on a CUDA device (sm_100a kernels only).")
        self.batch_size = int(batch_size)
        self.steps = int(steps)
        self.vocab_size = int(vocab_size)
        self.alpha_values = [float(x) for x in alpha_values]
        self.beta_values = [float(x) for x in beta_values]
        self.rank = int(local_head.lm_head_weight.shape[1])
        self._r = ops.round8(self.rank)  # carried rank width, zero-padded to a multiple of 8
        self.embedding_weight = ops.zero_pad(local_head.embedding_weight.detach().to(device=device).contiguous(),
                                             cols=self._r)
        self.lm_head_weight = ops.zero_pad(local_head.lm_head_weight.detach().to(device=device).contiguous(),
                                           cols=self._r)
        self._can_triton_fuse = True
        dtype = self.lm_head_weight.dtype
        if dtype != torch.bfloat16:
            raise ValueError(f"MarkovDeLSGraphRunner kernels are bf16; the local head is {dtype}.")

        baseline_flat = torch.zeros(self.vocab_size, dtype=dtype, device=device)
        if baseline_logits is not None:
            baseline_numel = int(baseline_logits.numel())
            if baseline_numel != self.vocab_size:
                raise ValueError(
                    "Markov DeLS graph baseline vocab size mismatch: "
                    f"baseline={baseline_numel}, vocab={self.vocab_size}."
                )
            baseline_flat.copy_(baseline_logits.to(device=device, dtype=dtype).reshape(-1))
        self.baseline_logits = baseline_flat.contiguous()
        self.has_baseline = baseline_logits is not None
        self._prior_f32 = self.baseline_logits.to(torch.float32) if self.has_baseline else None

        B, S = self.batch_size, self.steps
        self.static_prev_ids = torch.zeros(B, 1, dtype=torch.long, device=device)
        self.static_base_logits = torch.zeros(B, S, self.vocab_size, dtype=dtype, device=device)
        self.static_out = torch.zeros(B, S, dtype=torch.long, device=device)
        self._alpha = torch.tensor(self.alpha_values, dtype=torch.float32, device=device)
        self._beta = torch.tensor(self.beta_values, dtype=torch.float32, device=device)
        self._tokens = torch.zeros(S, B, dtype=torch.long, device=device)
        self._s_scaled = torch.zeros(B, self._r, dtype=dtype, device=device)
        self._step_keys = torch.empty(S, B, dtype=torch.int64, device=device)  # one key slot per step
        self._ws = ops.Workspace(1 << 12, device)
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

    def _forward_impl(self):
        current = self.static_prev_ids[:, 0]
        for step in range(self.steps):
            # the gather resets this step's key slot; from the second step on it reads the
            # previous step's packed keys
            ops.gather_scaled_rows(current, self.embedding_weight, self._alpha[step : step + 1], self._s_scaled,
                                   keys=self._step_keys[step], ws=self._ws, tokens_are_keys=step > 0)
            ops.fused_argmax_base_bf16(
                self.static_base_logits[:, step, :], self._s_scaled, self.lm_head_weight, self._prior_f32,
                self._beta[step : step + 1], n_pos=1, keys_ready=True, out=self._key_outs[step], ws=self._ws,
            )
            current = self._step_keys[step]
        ops.keys_decode(self._step_keys.view(-1), tokens=self._tokens.view(-1), with_scores=False)
        self.static_out.copy_(self._tokens.t())

    @torch.inference_mode()
    def __call__(
        self,
        prev_token_ids: torch.Tensor,
        base_logits: torch.Tensor,
    ) -> torch.Tensor:
        self.static_prev_ids.copy_(prev_token_ids)
        self.static_base_logits.copy_(base_logits)
        self.graph.replay()
        return self.static_out.clone()
