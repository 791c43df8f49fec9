"""Gemma3 attention projections (kappa/gemma3/linear.py:9-23) with W8 weights.

kappa's Gemma3 projections take full-precision weights; the W8 form uses
Qwen3's ``Q8Weight`` as the Gemma3 MLP does.  ``kv_w`` is the stacked
``[2, num_kv, model_dim, head_dim]`` weight; K and V are two ``kw8_linear``
calls on its two halves.
"""

from __future__ import annotations

import torch

from kappa_b200 import _dense
from kappa_b200.qwen3.linear import project_attn_out, project_q
from kappa_b200.qwen3.quant import Weight, kmajor

__all__ = ["project_q", "project_kv", "project_attn_out"]


def project_kv(x: torch.Tensor, kv_w: Weight) -> tuple[torch.Tensor, torch.Tensor]:
    """kappa/gemma3/linear.py:15-19: ``kv_w`` ``[2, num_kv, D, head_dim]`` -> k, v ``[B, T, num_kv, head_dim]``."""
    km = kmajor(kv_w, -2, "kv_w")
    if len(km.shape) != 4 or int(km.shape[0]) != 2:
        raise ValueError(f"kv_w must be [2, num_kv, model_dim, head_dim], got {tuple(kv_w.values.shape)}")
    _, nkv, h, d = (int(s) for s in km.shape)
    _dense.check_x(x, d)
    b, t = int(x.shape[0]), int(x.shape[1])
    x2 = x.reshape(b * t, d)
    k, v = (_dense.linear(x2, km.group(j)).reshape(b, t, nkv, h) for j in (0, 1))
    return k, v
