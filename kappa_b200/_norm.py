"""RMSNorm and the fused FFN sub-block shared by the Gemma3 and Qwen3 drop-ins."""

from __future__ import annotations

import torch

from kappa_b200 import _lib

_SCALE_DT = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16}


def _scale(s: torch.Tensor, d: int, name: str) -> torch.Tensor:
    _lib.require_cuda(s, name)
    if s.dtype not in _SCALE_DT:
        raise ValueError(f"{name}: scale dtype {s.dtype} unsupported")
    if s.numel() != d:
        raise ValueError(f"{name}: {s.numel()} values for {d} features")
    return s.reshape(d).contiguous()


def rms_norm(x: torch.Tensor, scale: torch.Tensor, *, kind: int, epsilon: float,
             out_dtype: torch.dtype | None) -> torch.Tensor:
    """``kw8_rms_norm`` over the last axis of bf16 ``x``."""
    _lib.require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or out_dtype not in (None, torch.bfloat16):
        raise ValueError("rms_norm: the W8 path keeps activations in bfloat16")
    d = int(x.shape[-1])
    s = _scale(scale, d, "scale")
    xc = x.contiguous()
    out = torch.empty_like(xc)
    T = xc.numel() // d if d else 0
    _lib.check(_lib.load().kw8_rms_norm(xc.data_ptr(), T, d, s.data_ptr(), _SCALE_DT[s.dtype], kind,
                                        float(epsilon), out.data_ptr(), _lib.stream_of(x)))
    return out


def block_norms(pre: torch.Tensor, post: torch.Tensor | None, d: int, kind: int, epsilon: float):
    """(kw8_block_norms, tensors to keep alive)."""
    p = _scale(pre, d, "pre-FFN norm scale")
    q = None
    if post is not None:
        q = _scale(post, d, "post-FFN norm scale").to(p.dtype)
    n = _lib.KW8BlockNorms(p.data_ptr(), None if q is None else q.data_ptr(), _SCALE_DT[p.dtype], kind,
                           float(epsilon))
    return n, (p, q)


def dense_block(h: torch.Tensor, gate, up, down, *, hidden: int, act: int, pre, post, kind: int,
                epsilon: float, keep) -> torch.Tensor:
    """``h + post(FFN(pre(h)))`` through ``kw8_dense_block``."""
    import ctypes

    b, t, d = h.shape
    hc = h.contiguous()
    T = b * t
    norms, keep_n = block_norms(pre, post, d, kind, epsilon)
    lib = _lib.load()
    out = torch.empty_like(hc)
    ws = torch.empty(int(lib.kw8_dense_block_workspace_size(T, d, hidden)), dtype=torch.uint8, device=h.device)
    _lib.check(lib.kw8_dense_block(hc.data_ptr(), T, d, hidden, gate, up, down, act, ctypes.byref(norms),
                                   out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(h)))
    del keep, keep_n
    return out

