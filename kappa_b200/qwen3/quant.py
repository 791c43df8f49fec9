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
    "Q8Tiled",
    "pack_weight",
    "unpack_weight",
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
    """A W8 weight as the kernels take it: int8 values K-major ``[.., N, K]``
    (or pre-packed, ``layout == LAYOUT_TILED``) + flat scales."""

    q: torch.Tensor  # [..., N, K] contiguous int8, or the tiled uint8 buffer
    scale: torch.Tensor  # flat: 1 value or prod(lead) * N values
    per_channel: bool
    shape: tuple = ()  # the K-major logical shape [..., N, K]
    layout: int = _lib.LAYOUT_KMAJOR

    def struct(self, offset_rows: int = 0) -> _lib.KW8Weight:
        """kw8_weight for rows [offset_rows, ...) of the [-1, K] view."""
        K = int(self.shape[-1])
        if self.layout == _lib.LAYOUT_TILED:
            if offset_rows % 16 or (offset_rows and int(self.shape[-2]) % 16):
                raise ValueError("tiled weights split only at 16-row tile boundaries")
            steps = (K + 127) // 128 * 2
            q_ptr = self.q.data_ptr() + (offset_rows // 16) * steps * 1024
        else:
            q_ptr = self.q.data_ptr() + offset_rows * K
        s_ptr = self.scale.data_ptr()
        if self.per_channel:
            s_ptr += offset_rows * self.scale.element_size()
        return _lib.KW8Weight(q_ptr, s_ptr, _DT[self.scale.dtype], int(self.per_channel), int(self.layout), 0)

    def group(self, j: int, count: int = 1) -> "KMajor":
        """Leading-axis groups [j, j + count) (weights stacked on axis 0)."""
        per = 1
        for d in self.shape[1:-2]:
            per *= int(d)
        rows = per * int(self.shape[-2])
        scale = self.scale[j * rows:(j + count) * rows] if self.per_channel else self.scale
        shape = (count,) + tuple(self.shape[1:]) if count != 1 else tuple(self.shape[1:])
        if self.layout == _lib.LAYOUT_TILED:
            q = self.q[j * per:(j + count) * per]
        else:
            q = self.q[j:j + count] if count != 1 else self.q[j]
        return KMajor(q=q, scale=scale, per_channel=self.per_channel, shape=shape, layout=self.layout)


class Q8Tiled(NamedTuple):
    """A W8 weight pre-packed for the kernels (``pack_weight``): the same int8
    values and scale as the ``Q8Weight`` it came from, stored in the tiled
    layout (``kw8_pack_weight``) that every kernel reads in whole contiguous
    pieces.  ``kshape`` is the K-major logical shape ``[.., N, K]`` and
    ``in_axis`` the contraction axis of kappa's logical shape."""

    tiled: torch.Tensor  # uint8 [groups, ceil(N / 16), steps, 1024]
    scale: torch.Tensor
    kshape: tuple
    in_axis: int

    @property
    def values_shape(self) -> tuple:
        s = tuple(self.kshape)
        return s[:-2] + (s[-1], s[-2]) if self.in_axis == -2 else s


_warned_layout = False


def kmajor(w: Weight, in_axis: int, name: str = "weight") -> KMajor:
    """View a W8 weight K-major; copies only if ``values`` is stored otherwise.

    A ``Q8Tiled`` weight is passed through in its packed layout.
    """
    global _warned_layout
    if isinstance(w, Q8Tiled):
        if _norm_axis(in_axis, len(w.kshape)) != w.in_axis:
            raise ValueError(f"{name}: packed with contraction axis {w.in_axis}, used with {in_axis}")
        _lib.require_cuda(w.tiled, name)
        s = w.scale
        per_channel = s.numel() > 1
        s = s.contiguous().reshape(-1) if per_channel else s.reshape(1).contiguous()
        return KMajor(q=w.tiled, scale=s, per_channel=per_channel, shape=tuple(int(d) for d in w.kshape),
                      layout=_lib.LAYOUT_TILED)
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
    return KMajor(q=q, scale=s, per_channel=per_channel, shape=tuple(int(d) for d in q.shape))


def to_compute_dtype(w: Weight, dtype: torch.dtype, *, in_axis: int = -2) -> torch.Tensor:
    """kappa/qwen3/quant.py:34-38: ``values.astype(dt) * scale.astype(dt)``.

    W8 weights are dequantised by the ``kw8_dequantize`` kernel (one rounding
    per product, as kappa); full-precision weights are cast.
    """
    if isinstance(w, Q8Tiled):
        return to_compute_dtype(unpack_weight(w), dtype, in_axis=w.in_axis)
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


def pack_weight(w: Weight, *, in_axis: int = -2) -> Q8Tiled:
    """Pre-pack a W8 weight into the tiled layout (``kw8_pack_weight``).

    The load-time step after ``quantize_weight`` (kappa quantises its whole
    parameter tree at load, kappa/qwen3/weights.py:143-170): the values and
    scales are unchanged, only their storage order differs, so every kernel
    reads whole contiguous pieces of the weights (512 bytes per warp load in
    the decode kernel).  ``in_axis`` is the contraction axis as for
    ``kmajor``.  Every FFN, MoE, linear and block function of this package
    accepts the result wherever it takes a ``Q8Weight``.
    """
    km = kmajor(w, in_axis)
    if km.layout == _lib.LAYOUT_TILED:
        return w
    K, N = int(km.shape[-1]), int(km.shape[-2])
    groups = km.q.numel() // (N * K)
    lib = _lib.load()
    nbytes = int(lib.kw8_packed_weight_bytes(groups, N, K))
    steps = (K + 127) // 128 * 2
    tiled = torch.empty((groups, (N + 15) // 16, steps, 1024), dtype=torch.uint8, device=km.q.device)
    assert tiled.numel() == nbytes
    _lib.check(lib.kw8_pack_weight(km.q.data_ptr(), groups, N, K, tiled.data_ptr(), _lib.stream_of(km.q)))
    return Q8Tiled(tiled=tiled, scale=w.scale, kshape=tuple(km.shape), in_axis=_norm_axis(in_axis, len(km.shape)))


def unpack_weight(w: Q8Tiled) -> Q8Weight:
    """The ``Q8Weight`` a ``Q8Tiled`` was packed from (values K-major in memory,
    kappa's logical shape), bit for bit."""
    kshape = tuple(w.kshape)
    K, N = kshape[-1], kshape[-2]
    groups = 1
    for d in kshape[:-2]:
        groups *= int(d)
    q = torch.empty(kshape, dtype=torch.int8, device=w.tiled.device)
    _lib.check(_lib.load().kw8_unpack_weight(w.tiled.data_ptr(), groups, N, K, q.data_ptr(), _lib.stream_of(q)))
    values = q.transpose(-1, -2) if w.in_axis == -2 else q
    return Q8Weight(values=values, scale=w.scale)
