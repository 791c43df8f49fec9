"""Attention projections (kappa/qwen3/linear.py:11-25) as W8 linears.

Same signatures and layouts as kappa: ``q_w`` / ``k_w`` / ``v_w``
``[heads, model_dim, head_dim]``, ``o_w`` ``[heads, head_dim, model_dim]``.
Each projection is one ``kw8_linear`` call (the tensor-core GEMM for
prefill, the weight-streaming kernel for decode) on the weight viewed
K-major: ``[heads * head_dim, model_dim]`` for Q/K/V (the storage
``quantize_weight`` produces for ``in_axis=-2``) and ``[model_dim, heads *
head_dim]`` for O (the storage :func:`quantize_attn_out` produces).
kappa computes ``einsum(x, to_compute_dtype(w, x.dtype))``: a bf16 product
of bf16 dequantised weights; here the int8 values are widened exactly, the
products accumulate in fp32 and the scale is applied to the sum.
"""

from __future__ import annotations

import torch

from kappa_b200 import _dense
from kappa_b200.qwen3.quant import KMajor, Q8Weight, Weight, is_q8_weight, kmajor, quantize_weight

__all__ = ["project_q", "project_kv", "project_attn_out", "quantize_attn_out", "attn_out_kmajor"]


def _project_heads(x: torch.Tensor, w: Weight, name: str) -> torch.Tensor:
    """``einsum("btd,ndh->btnh", x, w)`` for a W8 ``w`` ``[n, d, h]``."""
    km = kmajor(w, -2, name)
    if len(km.shape) != 3:
        raise ValueError(f"{name} must be [heads, model_dim, head_dim], got {tuple(w.values.shape)}")
    n, h, d = (int(s) for s in km.shape)
    _dense.check_x(x, d)
    b, t = int(x.shape[0]), int(x.shape[1])
    return _dense.linear(x.reshape(b * t, d), km).reshape(b, t, n, h)


def project_q(x: torch.Tensor, q_w: Weight) -> torch.Tensor:
    """kappa/qwen3/linear.py:11-13: ``q_w`` ``[num_heads, model_dim, head_dim]``."""
    return _project_heads(x, q_w, "q_w")


def project_kv(x: torch.Tensor, k_w: Weight, v_w: Weight) -> tuple[torch.Tensor, torch.Tensor]:
    """kappa/qwen3/linear.py:16-20: ``k_w``, ``v_w`` each ``[num_kv, model_dim, head_dim]``."""
    return _project_heads(x, k_w, "k_w"), _project_heads(x, v_w, "v_w")


def attn_out_kmajor(o_w: Weight) -> KMajor:
    """``o_w`` ``[n, h, d]`` as the K-major ``[d, n*h]`` weight of the output projection.

    A per-channel scale must hold one value per model-dim channel (the form
    :func:`quantize_attn_out` makes); values stored otherwise are copied.
    """
    if not is_q8_weight(o_w):
        raise TypeError("o_w: kappa_b200 implements the W8 path; quantize the weight first")
    v = o_w.values
    if v.dim() != 3:
        raise ValueError(f"o_w must be [heads, head_dim, model_dim], got {tuple(v.shape)}")
    n, h, d = (int(s) for s in v.shape)
    s = o_w.scale
    if s.numel() not in (1, d):
        raise ValueError(
            f"o_w: per-channel scales must be one per model-dim channel ({d}), got {s.numel()} "
            "(quantize the output projection with quantize_attn_out)"
        )
    flat = Q8Weight(values=v.reshape(n * h, d), scale=s.reshape(1, d) if s.numel() == d else s.reshape(()))
    return kmajor(flat, -2, "o_w")


def project_attn_out(encoded: torch.Tensor, o_w: Weight) -> torch.Tensor:
    """kappa/qwen3/linear.py:23-25: ``einsum("btnh,nhd->btd", encoded, o_w)``."""
    km = attn_out_kmajor(o_w)
    d, nh = (int(s) for s in km.shape)
    if encoded.dim() != 4 or int(encoded.shape[2]) * int(encoded.shape[3]) != nh:
        raise ValueError(f"encoded {tuple(encoded.shape)} does not match o_w {tuple(o_w.values.shape)}")
    b, t = int(encoded.shape[0]), int(encoded.shape[1])
    x = encoded.reshape(b, t, nh)
    _dense.check_x(x, nh)
    return _dense.linear(x.reshape(b * t, nh), km).reshape(b, t, d)


def quantize_attn_out(o_w: torch.Tensor, *, scale_dtype: torch.dtype = torch.bfloat16,
                      per_channel: bool = False) -> Q8Weight:
    """``quantize_weight`` of an output projection ``[n, h, d]`` over its whole
    contraction ``(n, h)``: per tensor this is kappa's result; per channel
    it gives one scale per model-dim channel.  ``values`` keeps the ``[n, h,
    d]`` shape as a view of the K-major ``[d, n*h]`` storage."""
    if o_w.dim() != 3:
        raise ValueError(f"o_w must be [heads, head_dim, model_dim], got {tuple(o_w.shape)}")
    n, h, d = (int(s) for s in o_w.shape)
    q = quantize_weight(o_w.reshape(n * h, d), scale_dtype=scale_dtype, per_channel=per_channel, in_axis=-2)
    scale = q.scale.reshape(1, 1, d) if per_channel else q.scale
    return Q8Weight(values=q.values.reshape(n, h, d), scale=scale)
