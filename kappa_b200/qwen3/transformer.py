"""The W8 embedding and LM head of kappa/qwen3/transformer.py:49-75.

``embed_tokens`` dequantises only the gathered rows (``kw8_embed_gather``);
the logits are one ``kw8_linear`` call over the ``[vocab, model_dim]`` head
(K-major as stored), the largest single weight read of a decode step.
``logits_from_hidden_last_positions`` gathers its rows inside the kernel.
"""

from __future__ import annotations

import torch

from kappa_b200 import _dense
from kappa_b200.qwen3.quant import Weight, gather_embed_tokens, is_q8_weight, kmajor

__all__ = ["embed_tokens", "logits_from_hidden", "logits_from_hidden_tied", "logits_from_hidden_last_positions"]


def embed_tokens(tokens: torch.Tensor, embed_table: Weight, *, compute_dtype: torch.dtype | None = None) -> torch.Tensor:
    """kappa/qwen3/transformer.py:49-52."""
    if compute_dtype is None:
        compute_dtype = embed_table.scale.dtype if is_q8_weight(embed_table) else embed_table.dtype
    return gather_embed_tokens(tokens, embed_table, compute_dtype=compute_dtype)


def _head(x: torch.Tensor, w: Weight, name: str, out_dtype: torch.dtype | None):
    km = kmajor(w, -1, name)
    if len(km.shape) != 2:
        raise ValueError(f"{name} must be [vocab, model_dim], got {tuple(w.values.shape)}")
    return km, (out_dtype or x.dtype)


def logits_from_hidden(x: torch.Tensor, lm_head: Weight, *, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """kappa/qwen3/transformer.py:55-59: ``einsum("btd,vd->btv")`` -> ``[B, T, vocab]``.

    kappa's result dtype is x's (bf16); ``out_dtype=torch.float32`` keeps
    the fp32 sums instead.
    """
    km, dt = _head(x, lm_head, "lm_head", out_dtype)
    V, D = (int(s) for s in km.shape)
    _dense.check_x(x, D)
    b, t = int(x.shape[0]), int(x.shape[1])
    return _dense.linear(x.reshape(b * t, D), km, out_dtype=dt).reshape(b, t, V)


def logits_from_hidden_tied(x: torch.Tensor, embed_table: Weight, *, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """kappa/qwen3/transformer.py:62-65 (the embedding table as the head)."""
    return logits_from_hidden(x, embed_table, out_dtype=out_dtype)


def logits_from_hidden_last_positions(x: torch.Tensor, w: Weight, last_idx: torch.Tensor, *,
                                      out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """kappa/qwen3/transformer.py:68-75: ``x`` ``[B, L, D]``, ``last_idx`` ``[B]`` -> ``[B, vocab]``."""
    km, dt = _head(x, w, "w", out_dtype)
    V, D = (int(s) for s in km.shape)
    _dense.check_x(x, D)
    b, L = int(x.shape[0]), int(x.shape[1])
    if tuple(last_idx.shape) != (b,):
        raise ValueError(f"last_idx must be [{b}], got {tuple(last_idx.shape)}")
    # JAX's gather: negative positions count from the end, then clamp into [0, L).
    li = last_idx.to(device=x.device, dtype=torch.int64)
    li = torch.where(li < 0, li + L, li).clamp(0, L - 1)
    rows = torch.arange(b, device=x.device, dtype=torch.int64) * L + li
    return _dense.linear(x.reshape(b * L, D), km, rows=rows, out_dtype=dt)
