"""Writes the golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

kappa (pure JAX) stores no golden arrays and cannot run here, so two kinds
of fixture pin the CPU oracle instead:

1. Known answers derived from kappa's documented semantics with exact
   rational arithmetic (``fractions.Fraction``), independent of NumPy's
   float ops:
     * ``quantize_weight`` (kappa/qwen3/quant.py:41-48): fp32 IEEE division
       ``amax / 127``, the FLT_MIN floor, ``w / scale`` rounded to fp32,
       round half to even, clip to [-128, 127], scale stored as bf16 (RNE);
     * ``jax.lax.top_k`` order (values descending, ties to the lower index)
       on hand-written logits;
     * the stable expert sort of ``_moe_ragged`` (kappa/qwen3/ffn_moe.py:196)
       and the fixed-capacity slots (ffn_moe.py:59-71) on hand-written ids.
2. Regression vectors: the oracle's outputs on small seeded inputs
   (``oracle_small.npz``), so GPU tests compare against committed numbers.
"""

from __future__ import annotations

import json
import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


# ---------------------------------------------------------------- exact ----


def round_to_format(q: Fraction, mant_bits: int, min_exp: int) -> Fraction:
    """Round a rational to the nearest binary float with ``mant_bits`` fraction
    bits (normal range exponent >= min_exp), ties to even."""
    if q == 0:
        return Fraction(0)
    sign = -1 if q < 0 else 1
    a = abs(q)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    e = max(e, min_exp)
    ulp = Fraction(2) ** (e - mant_bits)
    n = a / ulp
    fl = n.numerator // n.denominator
    rem = n - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return sign * fl * ulp


def to_f32(q: Fraction) -> Fraction:
    return round_to_format(q, 23, -126)


def to_bf16(q: Fraction) -> Fraction:
    return round_to_format(q, 7, -126)


def half_even(q: Fraction) -> int:
    fl = q.numerator // q.denominator
    rem = q - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return fl


FLT_MIN = Fraction(2) ** -126


def exact_quantize(ws: list[float], groups: list[list[int]]):
    """kappa's quantize over each index group (one group = per tensor)."""
    q = [0] * len(ws)
    scales = []
    for g in groups:
        amax = max(abs(Fraction(ws[i])) for i in g)
        s = max(to_f32(amax / 127), FLT_MIN)
        for i in g:
            r = half_even(to_f32(Fraction(ws[i]) / s))
            q[i] = min(127, max(-128, r))
        scales.append((s, to_bf16(s)))
    return q, scales


def quant_cases():
    cases = []

    def add(name, w, shape, per_channel_axis):
        arr = np.asarray(w, dtype=np.float32).reshape(shape)
        flat = [float(v) for v in arr.reshape(-1)]
        idx = np.arange(arr.size).reshape(shape)
        if per_channel_axis is None:
            groups = [list(range(arr.size))]
        else:
            moved = np.moveaxis(idx, per_channel_axis, -1)
            groups = [list(map(int, r)) for r in moved.reshape(-1, moved.shape[-1])]
        q, scales = exact_quantize(flat, groups)
        cases.append(
            {
                "name": name,
                "w": flat,
                "shape": list(shape),
                "per_channel_axis": per_channel_axis,
                "q": q,
                "scale_f32": [float(s) for s, _ in scales],
                "scale_bf16": [float(b) for _, b in scales],
            }
        )

    # amax 127 -> scale 1: exercises round half to even on exact .5 values.
    add("half_even", [0, 127, -127, 63.5, 64.5, -63.5, 0.5, 1.5, -0.5, 2.5, -2.5, 126.5], (3, 4), None)
    # amax 1 -> scale fl(1/127): w/scale lands next to .5 after fp32 rounding.
    add("inexact_scale", [1.0, -0.5, 0.25, 0.75, -1.0, 0.125, 0.0, -0.375], (2, 4), None)
    # all zero -> FLT_MIN floor, q = 0.
    add("zeros", [0.0] * 6, (2, 3), None)
    # tiny weights (scale just above FLT_MIN).
    add("tiny", [3e-36, -1e-36, 2e-36, 0.0], (2, 2), None)
    # per output channel (axis 0 = contraction for a [K, N] weight).
    add(
        "per_channel_k_axis0",
        [0.5, -2.0, 0.1, 3.0, -0.25, 1.0, 0.0, 0.2, -0.7, 6.0, 0.05, -0.4],
        (3, 4),
        0,
    )
    # per output channel, contraction on the last axis ([N, K] weight).
    add("per_channel_k_axis1", [1.0, 2.0, -3.0, 0.5, 0.25, -0.125, 10.0, -20.0, 5.0], (3, 3), 1)
    # 3-D stacked experts [E, K, N], contraction axis 1.
    add(
        "per_channel_stacked",
        [float(v) for v in np.linspace(-1.5, 2.25, 24, dtype=np.float32)],
        (2, 3, 4),
        1,
    )
    return cases


def topk_cases():
    # Hand-written logits and the jax.lax.top_k order (descending, ties to
    # the lower index), written out literally.
    return [
        {"logits": [[0.5, 2.0, 2.0, -1.0, 2.0, 0.0]], "k": 3, "idx": [[1, 2, 4]]},
        {"logits": [[1.0, 1.0, 1.0, 1.0]], "k": 2, "idx": [[0, 1]]},
        {"logits": [[-3.0, -1.0, -2.0, -1.0, 5.0]], "k": 4, "idx": [[4, 1, 3, 2]]},
        {"logits": [[0.0, -0.0, 0.25, 0.0]], "k": 3, "idx": [[2, 0, 1]]},
        {"logits": [[7.0, 3.0], [3.0, 7.0], [5.0, 5.0]], "k": 1, "idx": [[0], [1], [0]]},
    ]


def permute_cases():
    # idx [T, k] expert ids -> stable argsort of the flattened ids, bincount,
    # and each entry's slot within its expert, written out literally.
    return [
        {
            "idx": [[2, 0], [0, 1], [2, 1]],
            "E": 3,
            "order": [1, 2, 3, 5, 0, 4],
            "group_sizes": [2, 2, 2],
            "slot": [0, 0, 1, 0, 1, 1],
        },
        {
            "idx": [[3, 1], [3, 0], [3, 2], [1, 3]],
            "E": 5,
            "order": [3, 1, 6, 5, 0, 2, 4, 7],
            "group_sizes": [1, 2, 1, 4, 0],
            "slot": [0, 0, 1, 0, 2, 0, 1, 3],
        },
    ]


def oracle_small():
    sys.path.insert(0, ROOT)
    import oracle as O

    rng = np.random.default_rng(1234)
    out = {}
    # MoE: T=24 tokens, D=64, I=32, E=8, k=2.
    T, D, I, E, k = 24, 64, 32, 8, 2
    x = rng.standard_normal((1, T, D)).astype(np.float32).astype(O.BF16)
    router = (rng.standard_normal((D, E)) * 0.02).astype(np.float32)
    gate = (rng.standard_normal((E, D, I)) * 0.02).astype(np.float32)
    up = (rng.standard_normal((E, D, I)) * 0.02).astype(np.float32)
    down = (rng.standard_normal((E, I, D)) * 0.02).astype(np.float32)
    qr = O.quantize_weight(router, per_channel_axis=0, scale_dtype=np.float32)
    qg = O.quantize_weight(gate, per_channel_axis=1, scale_dtype=np.float32)
    qu = O.quantize_weight(up, per_channel_axis=1, scale_dtype=np.float32)
    qd = O.quantize_weight(down, per_channel_axis=1, scale_dtype=np.float32)
    x_flat, idx, w, b, t, d = O.route(x, qr, num_experts=E, num_experts_per_tok=k)
    y = O.moe_ragged(x_flat, idx, w, qg, qu, qd, num_experts=E, b=b, t=t, d=d)
    out.update(
        moe_x=x.view(np.uint16), moe_router=router, moe_gate=gate, moe_up=up, moe_down=down,
        moe_idx=idx, moe_w=w.view(np.uint16), moe_y=y.view(np.uint16),
        moe_shape=np.array([T, D, I, E, k]),
    )
    # Gemma-shaped MLP: T=16, D=64, H=128, gating [2, H, D], linear [H, D].
    T2, D2, H2 = 16, 64, 128
    x2 = rng.standard_normal((1, T2, D2)).astype(np.float32).astype(O.BF16)
    gating = (rng.standard_normal((2, H2, D2)) * 0.02).astype(np.float32)
    linear = (rng.standard_normal((H2, D2)) * 0.02).astype(np.float32)
    qgt = O.quantize_weight(gating, per_channel_axis=2, scale_dtype=np.float32)
    ql = O.quantize_weight(linear, per_channel_axis=0, scale_dtype=np.float32)
    y2 = O.feed_forward(x2, qgt, ql, transpose_gating_einsum=True)
    out.update(
        ffn_x=x2.view(np.uint16), ffn_gating=gating, ffn_linear=linear, ffn_y=y2.view(np.uint16),
        ffn_shape=np.array([T2, D2, H2]),
    )
    return out


def main() -> None:
    with open(os.path.join(HERE, "kat_quant.json"), "w") as f:
        json.dump(quant_cases(), f, indent=1)
    with open(os.path.join(HERE, "kat_topk.json"), "w") as f:
        json.dump(topk_cases(), f, indent=1)
    with open(os.path.join(HERE, "kat_permute.json"), "w") as f:
        json.dump(permute_cases(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), **oracle_small())
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
