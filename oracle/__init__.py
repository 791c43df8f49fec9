"""CPU oracle for the W8 feed-forward path — TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy (+ ml_dtypes for bf16 rounding), the
arithmetic of kappa's W8 fake-quant feed-forward functions.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it, and only as the checker or as the timed CPU baseline.  The
product package ``kappa_b200`` never imports it and has no CPU path.

Parity status: **unpinned against the reference's own outputs.**  kappa is
pure JAX; JAX is not installable here, and kappa's tests keep no golden
arrays (its checks draw inputs from ``jax.random``, which NumPy cannot
reproduce bit for bit).  The restatement is pinned instead by
  * hand-derived known answers of the documented semantics (round half to
    even, clip to [-128, 127], FLT_MIN scale floor, top-k ties to the lower
    index) in ``tests/golden/``;
  * kappa's own cross-checks restated on NumPy inputs:
    ``scripts/verify_qwen3_quant.py:13-25`` (W8 projection rel L2 <= 0.02) and
    ``scripts/verify_qwen3_moe_impls.py:49-117`` (gather == ragged ==
    high-capacity fixed, fp32, 1e-5 / 1e-4).
"""

from oracle.kappa_ref import (  # noqa: F401
    BF16,
    Q8Weight,
    bf16_round,
    feed_forward,
    gather_embed_tokens,
    gemma_ffn_sub_block,
    linear_f32,
    logits_from_hidden,
    logits_from_hidden_last_positions,
    project_attn_out,
    project_kv,
    project_q,
    qwen_dense_sub_block,
    qwen_moe_sub_block_f32,
    rms_norm,
    fixed_capacity_slots,
    fixed_capacity_value,
    moe_fixed_capacity,
    moe_gather_einsum,
    moe_ragged,
    moe_reference_f32,
    moe_swiglu_ffn,
    permute,
    quantize_weight,
    route,
    router_logits,
    swiglu_ffn,
    to_compute_dtype,
    topk_softmax,
)
