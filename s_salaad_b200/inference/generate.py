"""Greedy generation with a KV cache.

The reference's loop (``ssalaad/inference/generate.py:12-26``) recomputes the
whole prefix every step (``use_cache=False``), so every step runs the
compressed projections on ``batch x length`` tokens and a served model never
reaches the small-batch (decode) kernels.  :func:`generate` keeps the same
arguments, result and errors, but runs the prompt once (prefill, tensor-core
kernels from 128 tokens on) and then one token per sequence per step against
the attention KV cache, so each step's projections run on ``batch`` tokens
(the mma.sync decode kernels).  :func:`generate_no_cache` is the reference's
algorithm, kept for comparison and measurement.
"""
from __future__ import annotations

import torch


def _check_request(model, input_ids: torch.Tensor, max_new_tokens: int) -> None:
    """The reference's argument checks and messages (generate.py:14-19)."""
    if input_ids.ndim != 2 or input_ids.shape[1] == 0:
        raise ValueError("Expected a nonempty batch of input token IDs.")
    if max_new_tokens < 0:
        raise ValueError("max_new_tokens must be nonnegative.")
    if input_ids.shape[1] + max_new_tokens > model.config.max_position_embeddings:
        raise ValueError("Prompt and output exceed the configured context length.")


def _next_token(logits: torch.Tensor) -> torch.Tensor:
    """Greedy choice from the last position's logits [batch, vocab]."""
    if not torch.isfinite(logits).all():
        raise FloatingPointError("Non-finite inference logits.")
    return logits.argmax(-1, keepdim=True)


@torch.inference_mode()
def generate(model, input_ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
    """Greedy decoding of ``max_new_tokens`` tokens after ``input_ids``
    [batch, prompt]; returns [batch, prompt + max_new_tokens].  One model
    forward per new token, as in the reference: the prompt (with the cache
    filled), then each chosen token alone with the cache."""
    _check_request(model, input_ids, max_new_tokens)
    if max_new_tokens == 0:
        return input_ids
    out = model(input_ids=input_ids, use_cache=True)
    cache = out.past_key_values
    chosen = [_next_token(out.logits[:, -1])]
    for _ in range(max_new_tokens - 1):
        out = model(input_ids=chosen[-1], past_key_values=cache, use_cache=True)
        cache = out.past_key_values
        chosen.append(_next_token(out.logits[:, -1]))
    return torch.cat([input_ids, *chosen], dim=1)


@torch.inference_mode()
def generate_no_cache(model, input_ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
    """The reference's algorithm: every step runs the whole sequence again."""
    _check_request(model, input_ids, max_new_tokens)
    sequence = input_ids
    for _ in range(max_new_tokens):
        nxt = _next_token(model(input_ids=sequence, use_cache=False).logits[:, -1])
        sequence = torch.cat((sequence, nxt), dim=1)
    return sequence
