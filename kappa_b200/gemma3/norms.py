"""RMSNorm with Gemma's ``(1 + scale)`` (kappa/gemma3/norms.py:8-13) on the B200 kernel."""

from __future__ import annotations

import torch

from kappa_b200 import _lib, _norm


def rms_norm(x: torch.Tensor, scale: torch.Tensor, *, epsilon: float = 1e-6,
             out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * (1 + scale)`` in fp32, rounded to bf16."""
    return _norm.rms_norm(x, scale, kind=_lib.NORM_GEMMA, epsilon=epsilon, out_dtype=out_dtype)
