"""W8 weights: kappa/qwen3/quant.py on the B200 kernels.

``Q8Weight`` keeps kappa's meaning (int8 ``values`` with kappa's logical
shape, plus ``scale``; ``dequant = values * scale``).  Two things differ:

* ``quantize_weight`` also offers the per-output-channel form
  (``per_channel=True``: absmax over the contraction axis for every output
  channel, scales kept with a size-1 contraction axis so that
  ``values * scale`` still broadcasts);
* ``values`` is stored contraction-axis innermost ("K-major") as the
  tensor-core kernels read it.  For the default ``in_axis=-2`` (kappa's
  ``[.., K, N]`` layouts: Qwen3 linears, experts, router, Gemma's
  ``linear``) ``values`` is a transposed view of a ``[.., N, K]`` buffer;
  its shape and element values are exactly kappa's.
"""

from __future__ import annotations

from typing import NamedTuple, TypeAlias, TypeGuard

import torch

from kappa_b200 import _lib

__all__ = [
    "Q8Weight",
    "Weight",
    "is_q8_weight",
    "weight_param_dtype",
    "to_compute_dtype",
    "quantize_weight",
    "kmajor",
    "gather_embed_tokens",
]


class Q8Weight(NamedTuple):
    """kappa/qwen3/quant.py:15-19 — symmetric int8 values and their scale."""

    values: torch.Tensor
    scale: torch.Tensor


Weight: TypeAlias = torch.Tensor | Q8Weight


def is_q8_weight(w: Weight) -> TypeGuard[Q8Weight]:
    """kappa/qwen3/quant.py:25-26."""
    return isinstance(w, Q8Weight)


def weight_param_dtype(w: Weight) -> torch.dtype:
    """kappa/qwen3/quant.py:29-31."""
    return w.scale.dtype if is_q8_weight(w) else w.dtype


_DT = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16}


def _norm_axis(axis: int, ndim: int) -> int:
    a = axis if axis < 0 else axis - ndim
    if a not in (-1, -2):
        raise ValueError("the contraction axis must be one of the last two axes")
    return a


def quantize_weight(
    w: torch.Tensor,
    *,
    scale_dtype: torch.dtype = torch.bfloat16,
    per_channel: bool = False,
    in_axis: int = -2,
) -> Q8Weight:
    """kappa/qwen3/quant.py:41-48 (``per_channel=False``), on the GPU.

    ``scale = max(amax / 127, FLT_MIN)`` in fp32, ``values =
    clip(round_half_even(w / scale), -128, 127)`` with that fp32 scale, and
    the stored scale rounded to ``scale_dtype`` — bit for bit kappa's
    arithmetic.  ``per_channel=True`` takes the absmax over ``in_axis`` (the
    contraction axis) for every output channel.  ``in_axis`` also fixes the
    storage order (see the module docstring).
    """
    _lib.require_cuda(w, "w")
    if w.dtype not in _DT:
        raise ValueError(f"quantize_weight: unsupported weight dtype {w.dtype}")
    if scale_dtype not in _DT:
        raise ValueError(f"quantize_weight: unsupported scale dtype {scale_dtype}")
    if w.dim() < 2:
        raise ValueError("quantize_weight: weight must have at least 2 dims")
    ax = _norm_axis(in_axis, w.dim())
    lead = tuple(w.shape[:-2])
    outer = 1
    for s in lead:
        outer *= int(s)
    if ax == -2:
        K, N = int(w.shape[-2]), int(w.shape[-1])
    else:
        N, K = int(w.shape[-2]), int(w.shape[-1])
    w3 = w.reshape((outer,) + tuple(w.shape[-2:]))
    so = int(w3.stride(0))
    sk, sn = (int(w3.stride(1)), int(w3.stride(2))) if ax == -2 else (int(w3.stride(2)), int(w3.stride(1)))
    phys = torch.empty(lead + (N, K), dtype=torch.int8, device=w.device)
    n_scale = outer * N if per_channel else 1
    scale_phys = torch.empty(n_scale, dtype=scale_dtype, device=w.device)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_quantize_workspace_size(outer, N)), dtype=torch.uint8, device=w.device)
    _lib.check(
        lib.kw8_quantize(
            w3.data_ptr(), _DT[w.dtype], outer, K, N, so, sk, sn, int(per_channel), _DT[scale_dtype],
            phys.data_ptr(), scale_phys.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(w),
        )
    )
    values = phys.transpose(-1, -2) if ax == -2 else phys
    if per_channel:
        scale = scale_phys.reshape(lead + (N,)).unsqueeze(ax)
    else:
        scale = scale_phys.reshape(())
    return Q8Weight(values=values, scale=scale)


class KMajor(NamedTuple):
    """A W8 weight as the kernels take it: [.., N, K] int8 + flat scales."""

    q: torch.Tensor  # [..., N, K] contiguous int8
    scale: torch.Tensor  # flat: 1 value or prod(lead) * N values
    per_channel: bool

    def struct(self, offset_rows: int = 0) -> _lib.KW8Weight:
        """kw8_weight for rows [offset_rows, ...) of the [-1, K] view."""
        K = self.q.shape[-1]
        q_ptr = self.q.data_ptr() + offset_rows * K
        s_ptr = self.scale.data_ptr()
        if self.per_channel:
            s_ptr += offset_rows * self.scale.element_size()
        return _lib.KW8Weight(q_ptr, s_ptr, _DT[self.scale.dtype], int(self.per_channel))


_warned_layout = False


def kmajor(w: Weight, in_axis: int, name: str = "weight") -> KMajor:
    """View a W8 weight K-major; copies only if ``values`` is stored otherwise."""
    global _warned_layout
    if not is_q8_weight(w):
        raise TypeError(
            f"{name}: kappa_b200 implements the W8 path; quantize the weight with "
            "kappa_b200.qwen3.quant.quantize_weight first"
        )
    v = w.values
    _lib.require_cuda(v, name)
    if v.dtype != torch.int8:
        raise ValueError(f"{name}: values must be int8")
    ax = _norm_axis(in_axis, v.dim())
    q = v.transpose(-1, -2) if ax == -2 else v
    if not q.is_contiguous():
        if not _warned_layout:
            import warnings

            warnings.warn(
                f"{name}: W8 values are not stored contraction-axis innermost; copying per call "
                "(quantize with kappa_b200's quantize_weight to avoid it)",
                stacklevel=3,
            )
            _warned_layout = True
        q = q.contiguous()
    s = w.scale
    if s.dtype not in _DT:
        raise ValueError(f"{name}: scale dtype {s.dtype} unsupported")
    if s.device != v.device:
        raise ValueError(f"{name}: scale and values on different devices")
    per_channel = s.numel() > 1
    if per_channel:
        s2 = s.squeeze(ax) if s.dim() == v.dim() else s
        expected = q.numel() // q.shape[-1]
        if s2.numel() != expected:
            raise ValueError(f"{name}: scale has {s.numel()} values, expected 1 or {expected}")
        s = s2.contiguous().reshape(-1)
    else:
        s = s.reshape(1).contiguous()
    return KMajor(q=q, scale=s, per_channel=per_channel)


def to_compute_dtype(w: Weight, dtype: torch.dtype, *, in_axis: int = -2) -> torch.Tensor:
    """kappa/qwen3/quant.py:34-38: ``values.astype(dt) * scale.astype(dt)``.

    W8 weights are dequantised by the ``kw8_dequantize`` kernel (one rounding
    per product, as kappa); full-precision weights are cast.
    """
    if not is_q8_weight(w):
        return w.to(dtype)
    if dtype not in _DT:
        raise ValueError(f"to_compute_dtype: unsupported dtype {dtype}")
    km = kmajor(w, in_axis)
    out = torch.empty(km.q.shape, dtype=dtype, device=km.q.device)
    K = int(km.q.shape[-1])
    N = int(km.q.shape[-2])
    groups = km.q.numel() // (N * K) if km.q.numel() else 0
    if groups:
        _lib.check(
            _lib.load().kw8_dequantize(km.struct(), groups, N, K, _DT[dtype], out.data_ptr(), _lib.stream_of(out))
        )
    return out.transpose(-1, -2) if _norm_axis(in_axis, out.dim()) == -2 else out


def gather_embed_tokens(tokens: torch.Tensor, embed: Weight, *, compute_dtype: torch.dtype) -> torch.Tensor:
    """kappa/qwen3/quant.py:51-57 for a W8 table ``[vocab, model_dim]``.

    Only the gathered rows are dequantised: ``values[t].astype(dt) *
    scale.astype(dt)`` with one rounding per product (``kw8_embed_gather``).
    Ids follow JAX's gather: negative ids count from the end, then ids are
    clamped into ``[0, vocab)``.  A per-channel table has one scale per row.
    """
    if not is_q8_weight(embed):
        raise TypeError("embed: kappa_b200 implements the W8 path; quantize the table first")
    if compute_dtype not in _DT:
        raise ValueError(f"gather_embed_tokens: unsupported compute dtype {compute_dtype}")
    km = kmajor(embed, -1, "embed")
    if km.q.dim() != 2:
        raise ValueError(f"embed must be [vocab, model_dim], got {tuple(embed.values.shape)}")
    V, D = (int(s) for s in km.q.shape)
    _lib.require_cuda(tokens, "tokens")
    t = tokens.to(torch.int32).contiguous()
    out = torch.empty(tuple(tokens.shape) + (D,), dtype=compute_dtype, device=tokens.device)
    _lib.check(
        _lib.load().kw8_embed_gather(
            t.data_ptr(), t.numel(), km.struct(), V, D, _DT[compute_dtype], out.data_ptr(), _lib.stream_of(t)
        )
    )
    return out
