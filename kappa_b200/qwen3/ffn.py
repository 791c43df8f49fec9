"""Dense SwiGLU FFN (kappa/qwen3/ffn.py:12-22) on the W8 kernels."""

from __future__ import annotations

import torch

from kappa_b200 import _dense, _lib
from kappa_b200.qwen3.quant import Weight, kmajor


def swiglu_ffn(
    x: torch.Tensor,
    gate_w: Weight,
    up_w: Weight,
    down_w: Weight,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """``gate_w``, ``up_w``: ``[model_dim, intermediate]``; ``down_w``: ``[intermediate, model_dim]``."""
    g = kmajor(gate_w, -2, "gate_w")
    u = kmajor(up_w, -2, "up_w")
    dn = kmajor(down_w, -2, "down_w")
    inter, dim = int(g.shape[-2]), int(g.shape[-1])
    if tuple(u.shape) != (inter, dim) or tuple(dn.shape) != (dim, inter) or len(g.shape) != 2:
        raise ValueError("swiglu_ffn: weight shapes do not match [D, I], [D, I], [I, D]")
    _dense.check_x(x, dim)
    return _dense.dense_ffn(
        x, g.struct(), u.struct(), dn.struct(), hidden=inter, act=_lib.ACT_SILU, keep=(g, u, dn),
        out_dtype=out_dtype,
    )
