"""Gemma3 gated-GELU MLP (kappa/gemma3/ffn.py:10-26) with W8 weights.

Same signature and layouts as kappa's ``feed_forward``; the weights are
``Q8Weight`` (kappa's own Gemma3 weights are full precision, so the W8 form
borrows Qwen3's ``Q8Weight``, kappa/qwen3/quant.py:15-22).  The whole MLP
runs as two tensor-core kernels: gate/up with the GELU·up epilogue, then
the down projection.
"""

from __future__ import annotations

import torch

from kappa_b200 import _dense, _lib
from kappa_b200.qwen3.quant import Weight, kmajor


def feed_forward(
    x: torch.Tensor,
    gating_w: Weight,
    linear_w: Weight,
    *,
    transpose_gating_einsum: bool,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """``gating_w``: ``[2, hidden, embed]`` if ``transpose_gating_einsum`` else ``[2, embed, hidden]``.

    ``linear_w``: ``[hidden, embed]``.  ``x``: ``[B, T, embed]`` bf16.
    Returns ``gelu_tanh(x·G0) * (x·G1) · L`` as ``[B, T, embed]``.
    """
    g = kmajor(gating_w, -1 if transpose_gating_einsum else -2, "gating_w")
    lw = kmajor(linear_w, -2, "linear_w")
    if len(g.shape) != 3 or g.shape[0] != 2:
        raise ValueError(f"gating_w must be [2, ., .], got {tuple(gating_w.values.shape)}")
    hidden, embed = int(g.shape[1]), int(g.shape[2])
    if tuple(lw.shape) != (embed, hidden):
        raise ValueError(f"linear_w shape {tuple(linear_w.values.shape)} != ({hidden}, {embed})")
    _dense.check_x(x, embed)
    return _dense.dense_ffn(
        x, g.struct(0), g.struct(hidden), lw.struct(), hidden=hidden, act=_lib.ACT_GELU_TANH,
        keep=(g, lw), out_dtype=out_dtype,
    )
