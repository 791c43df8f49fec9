"""The FFN half of a Qwen3 decoder block (kappa/qwen3/block.py:68-81) in one call.

kappa runs ``h2 = rms_norm(h, pre_ffn_norm)``, then ``moe_swiglu_ffn`` (MoE
blocks) or ``swiglu_ffn`` (dense blocks), then ``h + out``, with bf16
results in between.  ``ffn_sub_block`` keeps those roundings and runs the
whole sub-block as one library call: ``kw8_moe_block`` (the pre-norm pass,
the MoE layer into its fp32 combine buffer, one pass per row that rounds it
and adds ``h``) or ``kw8_dense_block``.
"""

from __future__ import annotations

import ctypes

import torch

from kappa_b200 import _dense, _lib, _norm
from kappa_b200.qwen3 import ffn_moe
from kappa_b200.qwen3.quant import kmajor


def ffn_sub_block(h: torch.Tensor, pre_ffn_norm: torch.Tensor, ffn, *, cfg=None, epsilon: float = 1e-6) -> torch.Tensor:
    """``h + ffn(rms_norm(h, pre_ffn_norm))``.

    ``ffn`` is kappa's ``MoEFfnParams`` (``router``, ``gate_proj``,
    ``up_proj``, ``down_proj``; needs ``cfg``) or ``DenseFfnParams``
    (``gate_proj``, ``up_proj``, ``down_proj``), or any object with those
    fields.
    """
    _dense.check_x(h)
    b, t, d = (int(s) for s in h.shape)
    if hasattr(ffn, "router"):
        if cfg is None:
            raise ValueError("an MoE block needs cfg")
        return _moe_block(h, pre_ffn_norm, ffn, cfg=cfg, epsilon=epsilon)
    g = kmajor(ffn.gate_proj, -2, "gate_proj")
    u = kmajor(ffn.up_proj, -2, "up_proj")
    dn = kmajor(ffn.down_proj, -2, "down_proj")
    inter, dim = int(g.shape[-2]), int(g.shape[-1])
    if dim != d or tuple(u.shape) != (inter, dim) or tuple(dn.shape) != (dim, inter) or len(g.shape) != 2:
        raise ValueError("ffn_sub_block: weight shapes do not match [D, I], [D, I], [I, D]")
    return _norm.dense_block(h, g.struct(), u.struct(), dn.struct(), hidden=inter, act=_lib.ACT_SILU,
                             pre=pre_ffn_norm, post=None, kind=_lib.NORM_QWEN, epsilon=epsilon, keep=(g, u, dn))


def _moe_block(h, pre_ffn_norm, ffn, *, cfg, epsilon):
    if not cfg.use_moe:
        raise ValueError("moe_swiglu_ffn requires cfg.use_moe")
    b, t, d = (int(s) for s in h.shape)
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    impl = ffn_moe._effective_moe_impl(cfg, total_tokens=b * t)
    if impl not in ffn_moe._VALID_IMPLS:
        raise ValueError(f"unknown moe_impl: {impl!r}")
    capacity = None
    if impl == "fixed_capacity":
        if cfg.moe_capacity_factor <= 0:
            raise ValueError("fixed_capacity requires cfg.moe_capacity_factor > 0")
        capacity = ffn_moe.fixed_capacity(cfg, b * t)
    r = ffn_moe._router(ffn.router, d, e)
    g, u, dn, ne, i = ffn_moe._experts(ffn.gate_proj, ffn.up_proj, ffn.down_proj, d)
    if ne != e:
        raise ValueError(f"expert weights hold {ne} experts, config says {e}")
    T = b * t
    hc = h.contiguous()
    norms, keep = _norm.block_norms(pre_ffn_norm, None, d, _lib.NORM_QWEN, epsilon)
    lib = _lib.load()
    out = torch.empty_like(hc)
    ws = torch.empty(int(lib.kw8_moe_block_workspace_size(T, d, i, e, k)), dtype=torch.uint8, device=h.device)
    _lib.check(lib.kw8_moe_block(hc.data_ptr(), T, d, i, e, k, -1 if capacity is None else int(capacity),
                                 r.struct(), g.struct(), u.struct(), dn.struct(), ctypes.byref(norms), out.data_ptr(),
                                 ws.data_ptr(), ws.numel(), _lib.stream_of(h)))
    del keep, r, g, u, dn
    return out
