"""MoE SwiGLU FFN (kappa/qwen3/ffn_moe.py) on the B200 kernels.

One device pipeline serves every ``moe_impl``: router GEMM (fp32 logits),
top-k + softmax, stable expert permutation, row gather, grouped W8A16
gate/up GEMM with the SwiGLU epilogue, grouped down GEMM, weighted combine.
kappa's ``gather_einsum``, ``ragged_jax`` and ``ragged_tokamax`` compute the
same function (kappa's own check, scripts/verify_qwen3_moe_impls.py:83-99,
holds them equal); ``fixed_capacity`` adds the per-expert slot limit of
ffn_moe.py:130-141, applied in the permutation.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from kappa_b200 import _dense, _lib
from kappa_b200.qwen3.quant import KMajor, Weight, kmajor

# ffn_moe.py:20: upper bound on B*T behind the static fixed-capacity width.
_MOE_FIXED_CAP_MAX_BT = 8192

_VALID_IMPLS = ("gather_einsum", "fixed_capacity", "ragged_jax", "ragged_tokamax")


def _fixed_capacity_buffer_slots(cfg) -> int:
    """kappa/qwen3/ffn_moe.py:23-31."""
    if cfg.moe_fixed_capacity_slots is not None:
        return max(1, int(cfg.moe_fixed_capacity_slots))
    k, e = cfg.num_experts_per_tok, cfg.num_experts
    if e <= 0 or k <= 0:
        return 1
    cap = cfg.moe_capacity_factor * _MOE_FIXED_CAP_MAX_BT * k / e
    return max(1, int(math.ceil(cap)))


def fixed_capacity(cfg, bt: int) -> int:
    """Rows kept per expert by ``fixed_capacity`` (ffn_moe.py:135-141).

    ``c_dyn = max(1, round(f32(factor) * f32(bt*k) / f32(E)))`` (round half to
    even, fp32), limited by the static buffer depth.
    """
    k, e = cfg.num_experts_per_tok, cfg.num_experts
    c = np.float32(cfg.moe_capacity_factor) * np.float32(bt * k) / np.float32(e)
    c_dyn = max(1, int(np.rint(np.float32(c))))
    return min(c_dyn, _fixed_capacity_buffer_slots(cfg))


def _effective_moe_impl(cfg, *, total_tokens: int) -> str:
    """kappa/qwen3/ffn_moe.py:219-223."""
    impl = cfg.moe_impl
    if impl in ("ragged_jax", "ragged_tokamax") and total_tokens <= cfg.moe_ragged_decode_token_threshold:
        return "gather_einsum"
    return impl


def _router(router_w: Weight, d: int, num_experts: int) -> KMajor:
    r = kmajor(router_w, -2, "router_w")
    if tuple(r.shape) != (num_experts, d):
        raise ValueError(f"router_w shape {tuple(router_w.values.shape)} != ({d}, {num_experts})")
    return r


def _experts(ffn_gate: Weight, ffn_up: Weight, ffn_down: Weight, d: int):
    g = kmajor(ffn_gate, -2, "ffn_gate")
    u = kmajor(ffn_up, -2, "ffn_up")
    dn = kmajor(ffn_down, -2, "ffn_down")
    if len(g.shape) != 3:
        raise ValueError("expert weights must be [E, D, I] / [E, I, D]")
    e, i, dd = (int(s) for s in g.shape)
    if dd != d or tuple(u.shape) != (e, i, d) or tuple(dn.shape) != (e, d, i):
        raise ValueError(
            f"expert weight shapes {tuple(ffn_gate.values.shape)}, {tuple(ffn_up.values.shape)}, "
            f"{tuple(ffn_down.values.shape)} do not match [E, {d}, I], [E, {d}, I], [E, I, {d}]"
        )
    return g, u, dn, e, i


def route_logits(x: torch.Tensor, router_w: Weight, *, num_experts: int, num_experts_per_tok: int):
    """_route (ffn_moe.py:38-56) -> (logits [T, E] f32, idx [T, k] i32, w [T, k] bf16)."""
    _dense.check_x(x)
    b, t, d = x.shape
    r = _router(router_w, d, num_experts)
    T = b * t
    xc = x.contiguous()
    logits = torch.empty((T, num_experts), dtype=torch.float32, device=x.device)
    idx = torch.empty((T, num_experts_per_tok), dtype=torch.int32, device=x.device)
    w = torch.empty((T, num_experts_per_tok), dtype=torch.bfloat16, device=x.device)
    _lib.check(
        _lib.load().kw8_moe_route(
            xc.data_ptr(), T, d, num_experts, num_experts_per_tok, r.struct(), logits.data_ptr(),
            idx.data_ptr(), w.data_ptr(), _lib.stream_of(x),
        )
    )
    return logits, idx, w


def _route(x: torch.Tensor, router_w: Weight, *, num_experts: int, num_experts_per_tok: int):
    """kappa/qwen3/ffn_moe.py:38-56 -> (x_flat, idx, w, b, t, d)."""
    _, idx, w = route_logits(x, router_w, num_experts=num_experts, num_experts_per_tok=num_experts_per_tok)
    b, t, d = x.shape
    return x.reshape(b * t, d), idx, w, b, t, d


def topk_softmax(logits: torch.Tensor, k: int):
    """Top-k (ties to the lower index) + softmax of ffn_moe.py:51-52 on given fp32 logits."""
    _lib.require_cuda(logits, "logits")
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise ValueError("logits must be [T, E] float32")
    lg = logits.contiguous()
    T, E = lg.shape
    idx = torch.empty((T, k), dtype=torch.int32, device=lg.device)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=lg.device)
    _lib.check(_lib.load().kw8_moe_topk(lg.data_ptr(), T, E, k, idx.data_ptr(), w.data_ptr(), _lib.stream_of(lg)))
    return idx, w


def permute(idx: torch.Tensor, num_experts: int, capacity: int | None = None, *, single_block: bool = False):
    """Stable expert sort (ffn_moe.py:196-200) -> (sorted_token, inv_pos, group_sizes, group_offsets).

    Runs the multi-block sort (``kw8_moe_permute_ws``); ``single_block=True``
    runs the scratch-free one-block kernel (``kw8_moe_permute``) instead.
    """
    _lib.require_cuda(idx, "idx")
    if idx.dtype != torch.int32 or idx.dim() != 2:
        raise ValueError("idx must be [T, k] int32")
    ic = idx.contiguous()
    T, k = ic.shape
    m = T * k
    dev = ic.device
    sorted_token = torch.full((m,), -1, dtype=torch.int32, device=dev)
    inv_pos = torch.empty((m,), dtype=torch.int32, device=dev)
    sizes = torch.empty((num_experts,), dtype=torch.int32, device=dev)
    offsets = torch.empty((num_experts + 1,), dtype=torch.int32, device=dev)
    cap = -1 if capacity is None else int(capacity)
    lib = _lib.load()
    if single_block:
        _lib.check(
            lib.kw8_moe_permute(
                ic.data_ptr(), T, k, num_experts, cap, sorted_token.data_ptr(), inv_pos.data_ptr(),
                sizes.data_ptr(), offsets.data_ptr(), _lib.stream_of(ic),
            )
        )
    else:
        ws = torch.empty(int(lib.kw8_moe_permute_workspace_size(num_experts)), dtype=torch.uint8, device=dev)
        _lib.check(
            lib.kw8_moe_permute_ws(
                ic.data_ptr(), T, k, num_experts, cap, sorted_token.data_ptr(), inv_pos.data_ptr(),
                sizes.data_ptr(), offsets.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(ic),
            )
        )
    return sorted_token, inv_pos, sizes, offsets


def expert_ffn(xs: torch.Tensor, group_offsets: torch.Tensor, ffn_gate: Weight, ffn_up: Weight, ffn_down: Weight):
    """The three ragged_dots + SwiGLU of ffn_moe.py:202-210 on rows sorted by expert."""
    _lib.require_cuda(xs, "xs")
    if xs.dtype != torch.bfloat16 or xs.dim() != 2:
        raise ValueError("xs must be [rows, D] bf16")
    rows, d = xs.shape
    g, u, dn, e, i = _experts(ffn_gate, ffn_up, ffn_down, d)
    if group_offsets.dtype != torch.int32 or group_offsets.numel() != e + 1:
        raise ValueError("group_offsets must be [E+1] int32")
    xc = xs.contiguous()
    ys = torch.empty_like(xc)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_moe_expert_ffn_workspace_size(rows, d, i, e)), dtype=torch.uint8, device=xs.device)
    _lib.check(
        lib.kw8_moe_expert_ffn(
            xc.data_ptr(), rows, d, i, e, group_offsets.data_ptr(), g.struct(), u.struct(), dn.struct(),
            ys.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(xs),
        )
    )
    return ys


def combine(ys: torch.Tensor, inv_pos: torch.Tensor, w: torch.Tensor, d: int):
    """Unpermute + weighted sum over k (ffn_moe.py:212-215) -> [T, D] bf16."""
    T, k = w.shape
    out = torch.empty((T, d), dtype=torch.bfloat16, device=ys.device)
    _lib.check(
        _lib.load().kw8_moe_combine(
            ys.contiguous().data_ptr(), inv_pos.data_ptr(), w.contiguous().data_ptr(), T, k, d, out.data_ptr(),
            _lib.stream_of(ys),
        )
    )
    return out


def _moe_layer(x, router_w, ffn_gate, ffn_up, ffn_down, *, num_experts: int, k: int, capacity: int | None):
    _dense.check_x(x)
    b, t, d = x.shape
    r = _router(router_w, d, num_experts)
    g, u, dn, e, i = _experts(ffn_gate, ffn_up, ffn_down, d)
    if e != num_experts:
        raise ValueError(f"expert weights hold {e} experts, config says {num_experts}")
    T = b * t
    xc = x.contiguous()
    out = torch.empty((b, t, d), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_moe_ffn_workspace_size(T, d, i, e, k)), dtype=torch.uint8, device=x.device)
    _lib.check(
        lib.kw8_moe_ffn(
            xc.data_ptr(), T, d, i, e, k, -1 if capacity is None else int(capacity),
            r.struct(), g.struct(), u.struct(), dn.struct(), out.data_ptr(), ws.data_ptr(), ws.numel(),
            _lib.stream_of(x),
        )
    )
    return out


def moe_swiglu_ffn(
    x: torch.Tensor,
    router_w: Weight,
    ffn_gate: Weight,
    ffn_up: Weight,
    ffn_down: Weight,
    *,
    cfg,
) -> torch.Tensor:
    """MoE SwiGLU forward (kappa/qwen3/ffn_moe.py:226-299).

    Shapes: ``router_w`` ``[D, E]``; ``ffn_*`` ``[E, D, I]`` / ``[E, I, D]`` for gate/up/down.
    ``cfg`` is kappa's ``Qwen3Config`` or :class:`~kappa_b200.qwen3.architecture.MoEConfig`.
    """
    if not cfg.use_moe:
        raise ValueError("moe_swiglu_ffn requires cfg.use_moe")
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    b, t = int(x.shape[0]), int(x.shape[1])
    impl = _effective_moe_impl(cfg, total_tokens=b * t)
    if impl not in _VALID_IMPLS:
        raise ValueError(f"unknown moe_impl: {impl!r}")
    capacity = None
    if impl == "fixed_capacity":
        if cfg.moe_capacity_factor <= 0:
            raise ValueError("fixed_capacity requires cfg.moe_capacity_factor > 0")
        capacity = fixed_capacity(cfg, b * t)
    return _moe_layer(x, router_w, ffn_gate, ffn_up, ffn_down, num_experts=e, k=k, capacity=capacity)


def moe_swiglu_ffn_legacy(
    x: torch.Tensor,
    router_w: Weight,
    ffn_gate: Weight,
    ffn_up: Weight,
    ffn_down: Weight,
    *,
    num_experts: int,
    num_experts_per_tok: int,
) -> torch.Tensor:
    """kappa/qwen3/ffn_moe.py:302-316 (always the dropless gather formulation)."""
    return _moe_layer(x, router_w, ffn_gate, ffn_up, ffn_down, num_experts=num_experts, k=num_experts_per_tok, capacity=None)
