"""NumPy restatement of kappa's W8 feed-forward path (test infrastructure only).

Every function cites the kappa source it restates (paths relative to the
kappa project root).  JAX/XLA arithmetic is emulated as follows:
  * bf16 values are ``ml_dtypes.bfloat16``; an elementwise op on bf16 inputs
    is computed in fp32 and rounded to bf16 once (round to nearest even);
  * a bf16 ``einsum`` / ``dot`` is an fp32-accumulated product of the
    (exactly widened) bf16 inputs, rounded to bf16 at the end;
  * fp32 ops are IEEE fp32 (NumPy float32, no fast math).
The order of fp32 summation inside a dot is BLAS's, not XLA's; outputs are
compared with a tolerance, never bit for bit, except the integer results
(int8 values, top-k indices, permutation) which are exact.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import ml_dtypes
import numpy as np

BF16 = np.dtype(ml_dtypes.bfloat16)
F32 = np.dtype(np.float32)
FLT_MIN = np.float32(np.finfo(np.float32).tiny)


def bf16_round(a) -> np.ndarray:
    """Round to bf16 (RNE) and return as float32."""
    return np.asarray(a, dtype=np.float32).astype(BF16).astype(np.float32)


class Q8Weight(NamedTuple):
    """kappa/qwen3/quant.py:15-19 — int8 values + scale (``values * scale``).

    ``scale`` is a 0-d array (kappa's per-tensor form) or, for the
    per-output-channel form, an array that broadcasts against ``values``
    (the contraction axis kept with size 1).
    """

    values: np.ndarray
    scale: np.ndarray


def is_q8_weight(w) -> bool:
    """kappa/qwen3/quant.py:25-26."""
    return isinstance(w, Q8Weight)


def quantize_weight(w, *, scale_dtype=BF16, per_channel_axis: int | None = None) -> Q8Weight:
    """kappa/qwen3/quant.py:41-48, plus a per-output-channel variant.

    ``per_channel_axis=None`` is kappa's function: one absmax over the tensor.
    Otherwise the absmax is taken over the contraction axis
    ``per_channel_axis`` only (kept with size 1), giving one scale per output
    channel (and per expert for stacked weights).

    As in kappa, the int8 values are computed with the fp32 scale, and the
    stored scale is that fp32 scale rounded to ``scale_dtype``.
    """
    w_f = np.asarray(w, dtype=np.float32)
    if per_channel_axis is None:
        amax = np.max(np.abs(w_f)).astype(np.float32)
    else:
        amax = np.max(np.abs(w_f), axis=per_channel_axis, keepdims=True).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    scale = np.maximum(scale, FLT_MIN).astype(np.float32)
    q = np.clip(np.rint(w_f / scale), -128.0, 127.0).astype(np.int8)
    return Q8Weight(values=q, scale=np.asarray(scale).astype(scale_dtype))


def to_compute_dtype(w, dtype) -> np.ndarray:
    """kappa/qwen3/quant.py:34-38: ``values.astype(dt) * scale.astype(dt)``.

    For bf16 the product of two bf16 numbers is exact in fp32 and is rounded
    to bf16 once, which is what ``ml_dtypes`` does.  Returns ``dtype``.
    """
    dtype = np.dtype(dtype)
    if is_q8_weight(w):
        return w.values.astype(dtype) * np.asarray(w.scale).astype(dtype)
    return np.asarray(w).astype(dtype)


def _dot(a: np.ndarray, b: np.ndarray, dt) -> np.ndarray:
    """Dot in compute dtype ``dt``: fp32 accumulate, result rounded to ``dt``."""
    r = np.matmul(a.astype(np.float32), b.astype(np.float32))
    return r.astype(dt)


def _as(a, dt) -> np.ndarray:
    """Elementwise result computed in fp32, rounded to the compute dtype."""
    return np.asarray(a, dtype=np.float32).astype(dt).astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """jax.nn.gelu(x) with its default approximate=True, in fp32."""
    x = x.astype(np.float32)
    c = np.float32(math.sqrt(2.0 / math.pi))
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))).astype(
        np.float32
    )


def silu(x: np.ndarray) -> np.ndarray:
    """jax.nn.silu(x) = x * sigmoid(x), in fp32."""
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


# --------------------------------------------------------------------------
# dense FFNs
# --------------------------------------------------------------------------


def feed_forward(x, gating_w, linear_w, *, transpose_gating_einsum: bool, compute_dtype=BF16) -> np.ndarray:
    """kappa/gemma3/ffn.py:10-26 with W8 weights dequantised as quant.py:34-38.

    x [B, T, D] bf16; gating_w [2, H, D] (transpose) or [2, D, H]; linear_w [H, D].
    ``compute_dtype=BF16`` is kappa's arithmetic (bf16 einsums, bf16
    intermediates); ``np.float32`` is the fp32 dequantise-then-dot reference
    the parity bar is stated against (fp32 weights, intermediates and output).
    """
    dt = np.dtype(compute_dtype)
    x = np.asarray(x).astype(BF16).astype(dt)
    g = to_compute_dtype(gating_w, dt)
    lw = to_compute_dtype(linear_w, dt)
    if transpose_gating_einsum:
        gate = _dot(x, np.swapaxes(g[0], 0, 1), dt)
        up = _dot(x, np.swapaxes(g[1], 0, 1), dt)
    else:
        gate = _dot(x, g[0], dt)
        up = _dot(x, g[1], dt)
    a = (_as(gelu_tanh(gate.astype(np.float32)), dt) * up.astype(np.float32)).astype(dt)
    return _dot(a, lw, dt)


def swiglu_ffn(x, gate_w, up_w, down_w, *, compute_dtype=BF16) -> np.ndarray:
    """kappa/qwen3/ffn.py:12-22; weights [D, I], [D, I], [I, D] (see feed_forward for compute_dtype)."""
    dt = np.dtype(compute_dtype)
    x = np.asarray(x).astype(BF16).astype(dt)
    gate = _dot(x, to_compute_dtype(gate_w, dt), dt)
    up = _dot(x, to_compute_dtype(up_w, dt), dt)
    a = (_as(silu(gate.astype(np.float32)), dt) * up.astype(np.float32)).astype(dt)
    return _dot(a, to_compute_dtype(down_w, dt), dt)


# --------------------------------------------------------------------------
# MoE
# --------------------------------------------------------------------------


def router_logits(x_flat, router_w) -> np.ndarray:
    """kappa/qwen3/ffn_moe.py:46-50: fp32 logits of f32(x) · f32(dequant(router))."""
    rw = to_compute_dtype(router_w, F32)
    return np.matmul(np.asarray(x_flat).astype(np.float32), rw).astype(np.float32)


def topk_softmax(logits: np.ndarray, k: int, out_dtype=BF16) -> tuple[np.ndarray, np.ndarray]:
    """kappa/qwen3/ffn_moe.py:51-52.

    ``jax.lax.top_k``: the k largest values, in descending order, ties
    broken towards the lower index.  A stable sort of ``-logits`` gives
    exactly that order.  The weights are ``softmax`` over the k selected
    logits in fp32 (``exp(v - max) / sum``), cast to the activation dtype.
    """
    logits = np.asarray(logits, dtype=np.float32)
    order = np.argsort(-logits, axis=-1, kind="stable")[..., :k].astype(np.int32)
    top = np.take_along_axis(logits, order, axis=-1)
    m = np.max(top, axis=-1, keepdims=True)
    e = np.exp(top - m).astype(np.float32)
    w = (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return order, w.astype(out_dtype)


def route(x, router_w, *, num_experts: int, num_experts_per_tok: int):
    """kappa/qwen3/ffn_moe.py:38-56 -> (x_flat, idx, w, b, t, d)."""
    x = np.asarray(x)
    d = x.shape[-1]
    rw_shape = (router_w.values if is_q8_weight(router_w) else np.asarray(router_w)).shape
    if rw_shape != (d, num_experts):
        raise ValueError(f"router_w shape {rw_shape} != ({d}, {num_experts})")
    b, t, _ = x.shape
    x_flat = x.reshape(b * t, d)
    logits = router_logits(x_flat, router_w)
    idx, w = topk_softmax(logits, num_experts_per_tok, out_dtype=x.dtype)
    return x_flat, idx, w, b, t, d


def permute(idx: np.ndarray, num_experts: int, capacity: int | None = None):
    """Stable expert sort of kappa/qwen3/ffn_moe.py:189-200 (+ :130-141 slots).

    Returns (order, group_sizes, slot): ``order`` is the stable argsort of
    the flattened expert ids (rows kept by the capacity rule only),
    ``group_sizes`` the kept rows per expert, ``slot`` the position of each
    flat entry within its expert (ffn_moe.py:59-71).
    """
    expert_flat = np.asarray(idx, dtype=np.int32).reshape(-1)
    order = np.argsort(expert_flat, kind="stable").astype(np.int32)
    sorted_e = expert_flat[order]
    counts = np.bincount(sorted_e, minlength=num_experts).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    slot_sorted = np.arange(order.size) - starts[sorted_e]
    slot = np.empty_like(slot_sorted)
    slot[order] = slot_sorted
    if capacity is None:
        return order, counts.astype(np.int32), slot.astype(np.int32)
    keep_sorted = slot_sorted < capacity
    kept = np.bincount(sorted_e[keep_sorted], minlength=num_experts).astype(np.int32)
    return order[keep_sorted], kept, slot.astype(np.int32)


def _ragged_dot(lhs: np.ndarray, rhs: np.ndarray, group_sizes: np.ndarray) -> np.ndarray:
    """jax.lax.ragged_dot: rows of ``lhs`` in consecutive groups, group g times rhs[g]."""
    out = np.zeros((lhs.shape[0], rhs.shape[-1]), dtype=np.float32)
    start = 0
    for g, n in enumerate(np.asarray(group_sizes).tolist()):
        if n:
            out[start : start + n] = np.matmul(lhs[start : start + n], rhs[g])
        start += n
    return out


def moe_ragged(
    x_flat, idx, w, ffn_gate, ffn_up, ffn_down, *, num_experts: int, b: int, t: int, d: int,
    capacity: int | None = None, combine_dtype=None,
):
    """kappa/qwen3/ffn_moe.py:174-216 (``ragged_jax``): fp32 expert compute.

    The final scatter-add is in x's dtype in kappa (``.at[].add`` on a bf16
    buffer); here the k contributions of each token are added in flat order,
    each partial sum rounded, which is XLA-CPU's sequential scatter.
    ``combine_dtype=np.float32`` keeps the combine in fp32 and returns fp32:
    the fp32 dequantise-then-dot reference of the parity bar (kappa's cast
    of the expert outputs to x's dtype, ffn_moe.py:213, is then skipped
    too).  ``capacity``
    drops rows whose slot within their expert is >= capacity
    (ffn_moe.py:130-141), for comparing the fixed-capacity path.
    """
    k = idx.shape[-1]
    bt = b * t
    w_flat = np.asarray(w).reshape(-1)
    order, group_sizes, _ = permute(idx, num_experts, capacity)
    token_flat = np.repeat(np.arange(bt, dtype=np.int32), k)
    sorted_x = np.asarray(x_flat)[token_flat[order]].astype(np.float32)
    wg = to_compute_dtype(ffn_gate, F32)
    wu = to_compute_dtype(ffn_up, F32)
    wd = to_compute_dtype(ffn_down, F32)
    g = _ragged_dot(sorted_x, wg, group_sizes)
    u = _ragged_dot(sorted_x, wu, group_sizes)
    h = (silu(g) * u).astype(np.float32)
    y_sorted = _ragged_dot(h, wd, group_sizes)
    dt = np.dtype(combine_dtype) if combine_dtype is not None else np.asarray(x_flat).dtype
    y_orig = np.zeros((bt * k, d), dtype=np.float32)
    y_orig[order] = _as(y_sorted, dt)
    contrib = _as(y_orig * w_flat.astype(np.float32)[:, None], dt).reshape(bt, k, d)
    out = np.zeros((bt, d), dtype=np.float32)
    for j in range(k):
        out = _as(out + contrib[:, j], dt)
    return out.astype(dt).reshape(b, t, d)


def moe_gather_einsum(x_flat, idx, w, ffn_gate, ffn_up, ffn_down, *, b: int, t: int, d: int):
    """kappa/qwen3/ffn_moe.py:74-104 with moe_take_dequant (quant.py:60-76).

    Computes in x's dtype (bf16 or fp32): each token's k experts dequantised
    to that dtype, einsums with fp32 accumulation, SwiGLU, weighted sum over
    k.  The per-(token, expert) dots are batched by expert here; the
    arithmetic of each dot is the same.
    """
    x_flat = np.asarray(x_flat)
    dt = x_flat.dtype
    k = idx.shape[-1]
    bt = b * t
    wg = to_compute_dtype(ffn_gate, dt)
    wu = to_compute_dtype(ffn_up, dt)
    wd = to_compute_dtype(ffn_down, dt)
    e_count = wg.shape[0]
    idx_c = np.clip(np.asarray(idx), 0, e_count - 1)
    y_k = np.zeros((bt, k, d), dtype=np.float32)
    for e in np.unique(idx_c):
        tok, slot = np.nonzero(idx_c == e)
        xe = x_flat[tok]
        g = _dot(xe, wg[e], dt).astype(np.float32)
        u = _dot(xe, wu[e], dt).astype(np.float32)
        h = (_as(silu(g), dt) * u).astype(dt)
        y_k[tok, slot] = _dot(h, wd[e], dt).astype(np.float32)
    prod = _as(y_k * np.asarray(w).astype(np.float32)[..., None], dt)
    y = np.sum(prod, axis=1, dtype=np.float32).astype(dt)
    return y.reshape(b, t, d)


def fixed_capacity_slots(cfg, max_bt: int = 8192) -> int:
    """kappa/qwen3/ffn_moe.py:23-31."""
    if cfg.moe_fixed_capacity_slots is not None:
        return max(1, int(cfg.moe_fixed_capacity_slots))
    k, e = cfg.num_experts_per_tok, cfg.num_experts
    if e <= 0 or k <= 0:
        return 1
    return max(1, int(math.ceil(cfg.moe_capacity_factor * max_bt * k / e)))


def fixed_capacity_value(capacity_factor: float, bt: int, k: int, num_experts: int, slots: int) -> int:
    """kappa/qwen3/ffn_moe.py:135-141: rows kept per expert = min(c_dyn, c_buf)."""
    c_dyn = max(1, int(np.rint(np.float32(capacity_factor) * np.float32(bt * k) / np.float32(num_experts))))
    return min(c_dyn, int(slots))


def moe_fixed_capacity(
    x_flat, idx, w, ffn_gate, ffn_up, ffn_down, *, num_experts, capacity_factor, capacity_slots, b, t, d
):
    """kappa/qwen3/ffn_moe.py:107-158: token dropping by per-expert slot, in x's dtype."""
    k = idx.shape[-1]
    bt = b * t
    cap = fixed_capacity_value(capacity_factor, bt, k, num_experts, capacity_slots)
    _, _, slot = permute(idx, num_experts)
    valid = slot.reshape(bt, k) < cap
    x_flat = np.asarray(x_flat)
    dt = x_flat.dtype
    wg = to_compute_dtype(ffn_gate, dt)
    wu = to_compute_dtype(ffn_up, dt)
    wd = to_compute_dtype(ffn_down, dt)
    contrib = np.zeros((bt, k, d), dtype=np.float32)
    for e in np.unique(idx):
        tok, j = np.nonzero((idx == e) & valid)
        if tok.size == 0:
            continue
        xe = x_flat[tok]
        g = _dot(xe, wg[e], dt).astype(np.float32)
        u = _dot(xe, wu[e], dt).astype(np.float32)
        h = (_as(silu(g), dt) * u).astype(dt)
        ye = _dot(h, wd[e], dt).astype(np.float32)
        contrib[tok, j] = _as(ye * np.asarray(w)[tok, j].astype(np.float32)[:, None], dt)
    out = np.zeros((bt, d), dtype=np.float32)
    for j in range(k):
        out = _as(out + contrib[:, j], dt)
    return out.astype(dt).reshape(b, t, d)


def moe_swiglu_ffn(x, router_w, ffn_gate, ffn_up, ffn_down, *, cfg):
    """kappa/qwen3/ffn_moe.py:226-299 dispatch (``cfg`` duck-typed like Qwen3Config)."""
    if not cfg.use_moe:
        raise ValueError("moe_swiglu_ffn requires cfg.use_moe")
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    x_flat, idx, w, b, t, d = route(x, router_w, num_experts=e, num_experts_per_tok=k)
    impl = cfg.moe_impl
    if impl in ("ragged_jax", "ragged_tokamax") and b * t <= cfg.moe_ragged_decode_token_threshold:
        impl = "gather_einsum"
    if impl == "gather_einsum":
        return moe_gather_einsum(x_flat, idx, w, ffn_gate, ffn_up, ffn_down, b=b, t=t, d=d)
    if impl == "fixed_capacity":
        if cfg.moe_capacity_factor <= 0:
            raise ValueError("fixed_capacity requires cfg.moe_capacity_factor > 0")
        return moe_fixed_capacity(
            x_flat,
            idx,
            w,
            ffn_gate,
            ffn_up,
            ffn_down,
            num_experts=e,
            capacity_factor=cfg.moe_capacity_factor,
            capacity_slots=fixed_capacity_slots(cfg),
            b=b,
            t=t,
            d=d,
        )
    if impl in ("ragged_jax", "ragged_tokamax"):
        return moe_ragged(x_flat, idx, w, ffn_gate, ffn_up, ffn_down, num_experts=e, b=b, t=t, d=d)
    raise ValueError(f"unknown moe_impl: {impl!r}")


def moe_reference_f32(x, router_w, ffn_gate, ffn_up, ffn_down, *, num_experts: int, k: int,
                      capacity: int | None = None, idx=None, w=None):
    """The parity reference for a MoE layer: kappa's routing (fp32 logits,
    top-k, bf16 softmax weights) and fp32 dequantise-then-dot expert compute
    with an fp32 combine.  ``idx`` / ``w`` override the routing choice and
    its weights (to compare expert compute on another implementation's
    routing, checked separately); returns (y fp32 [B, T, D], idx, w)."""
    x = np.asarray(x)
    b, t, d = x.shape
    x_flat = x.reshape(b * t, d)
    if idx is None:
        logits = router_logits(x_flat, router_w)
        idx, ow = topk_softmax(logits, k, out_dtype=x.dtype)
    else:
        idx = np.asarray(idx, dtype=np.int32)
        ow = None
    if w is None:
        if ow is None:
            logits = router_logits(x_flat, router_w)
            top = np.take_along_axis(logits, idx, axis=-1)
            e = np.exp(top - top.max(-1, keepdims=True)).astype(np.float32)
            ow = (e / e.sum(-1, keepdims=True, dtype=np.float32)).astype(x.dtype)
        w = ow
    y = moe_ragged(x_flat, idx, w, ffn_gate, ffn_up, ffn_down, num_experts=num_experts, b=b, t=t, d=d,
                   capacity=capacity, combine_dtype=np.float32)
    return y, idx, w


# --------------------------------------------------------------------------
# Neighbours of the FFN: norms, attention projections, embedding, LM head
# --------------------------------------------------------------------------


def rms_norm(x, scale, *, gemma: bool, epsilon: float = 1e-6, out_dtype=None) -> np.ndarray:
    """kappa/gemma3/norms.py:8-13 (``gemma=True``: ``* (1 + scale)``) and
    kappa/qwen3/norms.py:10-16 (``gemma=False``: ``* scale``), in fp32,
    rounded to ``out_dtype`` (x's dtype by default)."""
    x = np.asarray(x)
    out_dtype = np.dtype(out_dtype) if out_dtype is not None else x.dtype
    xf = x.astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(var + np.float32(epsilon))).astype(np.float32)
    s = np.asarray(scale).astype(np.float32)
    g = (np.float32(1.0) + s) if gemma else s
    return ((xf * r).astype(np.float32) * g).astype(np.float32).astype(out_dtype)


def linear_f32(x2d, w_kmajor: Q8Weight) -> np.ndarray:
    """The fp32 dequantise-then-dot reference of one W8 linear layer:
    ``x [T, K] . dequant(w)^T`` with ``w`` K-major ``[N, K]`` (scale broadcast
    over K), fp32 throughout."""
    wf = to_compute_dtype(w_kmajor, F32)
    return np.matmul(np.asarray(x2d).astype(np.float32), wf.T).astype(np.float32)


def project_q(x, q_w, *, compute_dtype=BF16) -> np.ndarray:
    """kappa/qwen3/linear.py:11-13: ``einsum("btd,ndh->btnh", x, dequant(q_w))``."""
    dt = np.dtype(compute_dtype)
    w = to_compute_dtype(q_w, dt).astype(np.float32)
    return np.einsum("btd,ndh->btnh", np.asarray(x).astype(np.float32), w).astype(np.float32).astype(dt)


def project_kv(x, k_w, v_w, *, compute_dtype=BF16):
    """kappa/qwen3/linear.py:16-20."""
    return project_q(x, k_w, compute_dtype=compute_dtype), project_q(x, v_w, compute_dtype=compute_dtype)


def project_attn_out(encoded, o_w, *, compute_dtype=BF16) -> np.ndarray:
    """kappa/qwen3/linear.py:23-25: ``einsum("btnh,nhd->btd", encoded, dequant(o_w))``."""
    dt = np.dtype(compute_dtype)
    w = to_compute_dtype(o_w, dt).astype(np.float32)
    return np.einsum("btnh,nhd->btd", np.asarray(encoded).astype(np.float32), w).astype(np.float32).astype(dt)


def gather_embed_tokens(tokens, embed: Q8Weight, *, compute_dtype) -> np.ndarray:
    """kappa/qwen3/quant.py:51-57 for a W8 table ``[V, D]``: the gathered
    int8 rows times the scale, one rounding per product.  Ids follow JAX's
    gather (``embed.values[t]``): a negative id counts from the end, then
    ids are clamped into [0, V)."""
    dt = np.dtype(compute_dtype)
    V = embed.values.shape[0]
    t = np.asarray(tokens, dtype=np.int64)
    t = np.where(t < 0, t + V, t)
    t = np.clip(t, 0, V - 1)
    rows = embed.values[t]
    s = np.asarray(embed.scale)
    if s.ndim == embed.values.ndim:  # one scale per row
        s = s[t]
    return rows.astype(dt) * s.astype(dt)


def logits_from_hidden(x, lm_head: Q8Weight, *, compute_dtype=BF16) -> np.ndarray:
    """kappa/qwen3/transformer.py:55-59: ``einsum("btd,vd->btv")`` in x's dtype."""
    dt = np.dtype(compute_dtype)
    w = to_compute_dtype(lm_head, dt).astype(np.float32)
    return np.einsum("btd,vd->btv", np.asarray(x).astype(np.float32), w).astype(np.float32).astype(dt)


def logits_from_hidden_last_positions(x, w: Q8Weight, last_idx, *, compute_dtype=BF16) -> np.ndarray:
    """kappa/qwen3/transformer.py:68-75 (``x[rows, last_idx]`` with JAX's
    negative-index and clamping rules)."""
    x = np.asarray(x)
    b, L = x.shape[:2]
    li = np.asarray(last_idx, dtype=np.int64)
    li = np.clip(np.where(li < 0, li + L, li), 0, L - 1)
    h = x[np.arange(b), li]
    dt = np.dtype(compute_dtype)
    wf = to_compute_dtype(w, dt).astype(np.float32)
    return np.einsum("bd,vd->bv", h.astype(np.float32), wf).astype(np.float32).astype(dt)


def gemma_ffn_sub_block(h, pre_scale, gating_w, linear_w, post_scale=None, *, transpose_gating_einsum=True,
                        compute_dtype=BF16, epsilon: float = 1e-6) -> np.ndarray:
    """kappa/gemma3/block.py:73-82: ``h + rms_norm?(feed_forward(rms_norm(h, pre)))``
    with bf16 results between the steps (``compute_dtype`` as feed_forward)."""
    h = np.asarray(h)
    xn = rms_norm(h, pre_scale, gemma=True, epsilon=epsilon)
    out = feed_forward(xn, gating_w, linear_w, transpose_gating_einsum=transpose_gating_einsum,
                       compute_dtype=compute_dtype).astype(np.float32).astype(BF16)
    if post_scale is not None:
        out = rms_norm(out, post_scale, gemma=True, epsilon=epsilon)
    return (h.astype(np.float32) + out.astype(np.float32)).astype(BF16)


def qwen_dense_sub_block(h, pre_scale, gate_w, up_w, down_w, *, compute_dtype=BF16, epsilon: float = 1e-6):
    """kappa/qwen3/block.py:68-81 for a dense block: ``h + swiglu_ffn(rms_norm(h))``."""
    h = np.asarray(h)
    xn = rms_norm(h, pre_scale, gemma=False, epsilon=epsilon)
    out = swiglu_ffn(xn, gate_w, up_w, down_w, compute_dtype=compute_dtype).astype(np.float32).astype(BF16)
    return (h.astype(np.float32) + out.astype(np.float32)).astype(BF16)


def qwen_moe_sub_block_f32(h, pre_scale, router_w, ffn_gate, ffn_up, ffn_down, *, num_experts: int, k: int,
                           epsilon: float = 1e-6, idx=None, w=None):
    """kappa/qwen3/block.py:68-81 for an MoE block with the fp32 reference of
    the MoE layer (moe_reference_f32): the normed input is bf16, the layer
    output is rounded to bf16, then ``h +`` in bf16.  Returns (out, idx, w)."""
    h = np.asarray(h)
    xn = rms_norm(h, pre_scale, gemma=False, epsilon=epsilon)
    y, idx, w = moe_reference_f32(xn, router_w, ffn_gate, ffn_up, ffn_down, num_experts=num_experts, k=k,
                                  idx=idx, w=w)
    out = (h.astype(np.float32) + y.astype(BF16).astype(np.float32)).astype(BF16)
    return out, idx, w, xn
