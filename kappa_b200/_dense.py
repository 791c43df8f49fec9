"""Shared driver of the gated dense FFN kernels (Gemma3 MLP, Qwen3 SwiGLU)."""

from __future__ import annotations

import torch

from kappa_b200 import _lib
from kappa_b200.qwen3.quant import KMajor


def check_x(x: torch.Tensor, d: int | None = None) -> None:
    _lib.require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError(f"x must be [B, T, D], got shape {tuple(x.shape)}")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"x must be bfloat16 (the W8 path computes in bf16), got {x.dtype}")
    if d is not None and x.shape[-1] != d:
        raise ValueError(f"x feature dim {x.shape[-1]} != weight input dim {d}")


def dense_ffn(
    x: torch.Tensor,
    gate: _lib.KW8Weight,
    up: _lib.KW8Weight,
    down: _lib.KW8Weight,
    *,
    hidden: int,
    act: int,
    keep: tuple[KMajor, ...],
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """act(x·gateᵀ) * (x·upᵀ) · downᵀ through ``kw8_dense_ffn``.

    ``keep`` holds the tensors the kw8_weight structs point into, alive
    until the work is enqueued.
    """
    b, t, d = x.shape
    xc = x.contiguous()
    T = b * t
    lib = _lib.load()
    out = torch.empty((b, t, d), dtype=out_dtype, device=x.device)
    ws = torch.empty(int(lib.kw8_dense_ffn_workspace_size(T, d, hidden)), dtype=torch.uint8, device=x.device)
    _lib.check(
        lib.kw8_dense_ffn(
            xc.data_ptr(), T, d, hidden, gate, up, down, act,
            _lib.DT_F32 if out_dtype == torch.float32 else _lib.DT_BF16,
            out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(x),
        )
    )
    del keep
    return out


def linear(
    x2d: torch.Tensor,
    w: KMajor,
    *,
    rows: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """``x2d[r] . w^T`` through ``kw8_linear``: x2d ``[R, K]`` bf16, ``w`` K-major ``[N, K]``.

    With ``rows`` (int32 indices into x2d) the product runs on those rows
    only, gathered inside the kernel.  Returns ``[len(rows) or R, N]``.
    """
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out_dtype must be bfloat16 or float32, got {out_dtype}")
    K = int(w.shape[-1])
    if w.layout == _lib.LAYOUT_TILED and len(w.shape) > 2 and int(w.shape[-2]) % 16:
        raise ValueError("a stacked tiled weight is one linear layer only when its rows per group are a multiple of 16")
    N = 1
    for d in w.shape[:-1]:
        N *= int(d)
    xc = x2d.contiguous()
    if xc.dim() != 2 or int(xc.shape[1]) != K:
        raise ValueError(f"x rows have {tuple(xc.shape)[1:]} features, the weight takes {K}")
    T = int(xc.shape[0]) if rows is None else int(rows.numel())
    lib = _lib.load()
    out = torch.empty((T, N), dtype=out_dtype, device=x2d.device)
    ws = torch.empty(int(lib.kw8_linear_workspace_size(T, K, N)), dtype=torch.uint8, device=x2d.device)
    rows_c = None if rows is None else rows.to(torch.int32).contiguous()
    _lib.check(
        lib.kw8_linear(
            xc.data_ptr(), None if rows_c is None else rows_c.data_ptr(), T, K, N, w.struct(),
            _lib.DT_F32 if out_dtype == torch.float32 else _lib.DT_BF16, out.data_ptr(), ws.data_ptr(),
            ws.numel(), _lib.stream_of(x2d),
        )
    )
    del rows_c
    return out
