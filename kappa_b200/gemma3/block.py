"""The FFN half of a Gemma3 decoder block (kappa/gemma3/block.py:73-82) in one call.

kappa runs ``rms_norm(h, pre_ffw_norm_scale)`` -> ``feed_forward`` ->
``rms_norm(out, post_ffw_norm_scale)`` (when ``use_post_ffw_norm``) ->
``h + out`` as four XLA ops with bf16 results in between.  ``ffn_sub_block``
keeps those roundings and runs them as ``kw8_dense_block``: the pre-norm
pass, the gate/up GEMM, the down GEMM into fp32 partial sums, and one pass
per row that sums them, rounds, applies the post-norm and adds ``h``.
"""

from __future__ import annotations

import torch

from kappa_b200 import _dense, _lib, _norm
from kappa_b200.qwen3.quant import Weight, kmajor


def ffn_sub_block(
    h: torch.Tensor,
    pre_ffw_norm_scale: torch.Tensor,
    gating_weights: Weight,
    output_weights: Weight,
    post_ffw_norm_scale: torch.Tensor | None = None,
    *,
    transpose_gating_einsum: bool,
    epsilon: float = 1e-6,
) -> torch.Tensor:
    """``h + post_norm(feed_forward(rms_norm(h, pre)))``; ``post_ffw_norm_scale=None`` skips the post-norm."""
    g = kmajor(gating_weights, -1 if transpose_gating_einsum else -2, "gating_weights")
    lw = kmajor(output_weights, -2, "output_weights")
    if len(g.shape) != 3 or g.shape[0] != 2:
        raise ValueError(f"gating_weights must be [2, ., .], got {tuple(gating_weights.values.shape)}")
    hidden, embed = int(g.shape[1]), int(g.shape[2])
    if tuple(lw.shape) != (embed, hidden):
        raise ValueError(f"output_weights shape {tuple(output_weights.values.shape)} != ({hidden}, {embed})")
    _dense.check_x(h, embed)
    return _norm.dense_block(h, g.struct(0), g.struct(hidden), lw.struct(), hidden=hidden, act=_lib.ACT_GELU_TANH,
                             pre=pre_ffw_norm_scale, post=post_ffw_norm_scale, kind=_lib.NORM_GEMMA,
                             epsilon=epsilon, keep=(g, lw))
