"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Integer results (int8 values, scales, top-k indices, permutation) must be
bit exact; float outputs must meet the parity bar in helpers.parity
(max rel err 1e-2 plus a per-element bound) against the fp32
dequantise-then-dot reference, and a looser bound against kappa's own bf16
arithmetic (which carries its own rounding noise).
"""

from __future__ import annotations

import json
import os
from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle as O
from helpers import moe_weights, normal, parity, to_dev, to_np
from kappa_b200 import _lib
from kappa_b200.gemma3.ffn import feed_forward
from kappa_b200.qwen3 import ffn_moe as M
from kappa_b200.qwen3.architecture import MoEConfig
from kappa_b200.qwen3.ffn import swiglu_ffn
from kappa_b200.qwen3.quant import Q8Weight, quantize_weight, to_compute_dtype

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# Sanity bound against kappa's own bf16 arithmetic (bf16 intermediates and a
# bf16 scatter-add over k); the 1e-2 bar is checked against the fp32
# dequantise-then-dot reference.
KAPPA_BF16_TOL = 3e-2


_OPTS = (_lib.OPT_GEMM_PATH, _lib.OPT_TOKEN_TILE, _lib.OPT_DETERMINISTIC, _lib.OPT_TC_PAIR, _lib.OPT_EP_TIMING)


@pytest.fixture(autouse=True)
def _reset_options():
    for opt in _OPTS:
        _lib.set_option(opt, 0)
    yield
    for opt in _OPTS:
        _lib.set_option(opt, 0)
    if torch.cuda.is_available():
        dummy = torch.zeros(1, device="cuda")
        assert _lib.device_status(dummy) == 0, "a kernel reported a device-side error"


def _gpu_q(w: np.ndarray, per_channel: bool, in_axis: int = -2, scale_dtype=torch.float32) -> Q8Weight:
    return quantize_weight(to_dev(w), per_channel=per_channel, in_axis=in_axis, scale_dtype=scale_dtype)


def _oracle_q(w: np.ndarray, per_channel: bool, in_axis: int = -2, scale_dtype=np.float32) -> O.Q8Weight:
    return O.quantize_weight(w, per_channel_axis=(in_axis % w.ndim) if per_channel else None, scale_dtype=scale_dtype)


def _same_q(gq: Q8Weight, oq: O.Q8Weight):
    np.testing.assert_array_equal(to_np(gq.values), oq.values)
    gs = to_np(gq.scale)
    os_ = np.asarray(oq.scale)
    assert gs.shape == os_.shape, (gs.shape, os_.shape)
    np.testing.assert_array_equal(gs.astype(np.float32), os_.astype(np.float32))


# ------------------------------------------------------------ quantise ----


@pytest.mark.parametrize("case", json.load(open(os.path.join(GOLDEN, "kat_quant.json"))), ids=lambda c: c["name"])
def test_quantize_known_answers_gpu(case):
    w = np.asarray(case["w"], dtype=np.float32).reshape(case["shape"])
    ax = case["per_channel_axis"]
    in_axis = -2 if ax is None else ax - w.ndim
    if in_axis not in (-1, -2):
        pytest.skip("contraction axis must be one of the last two")
    g = quantize_weight(to_dev(w), per_channel=ax is not None, in_axis=in_axis)
    np.testing.assert_array_equal(to_np(g.values).reshape(-1), np.asarray(case["q"], dtype=np.int8))
    s = to_np(g.scale).astype(np.float32)
    if ax is not None:
        s = np.moveaxis(s, ax, -1)
    np.testing.assert_array_equal(s.reshape(-1), np.asarray(case["scale_bf16"], dtype=np.float32))


@pytest.mark.parametrize(
    "shape,in_axis,per_channel,src_dtype,scale_dtype",
    [
        ((4, 64, 48), -2, True, np.float32, torch.float32),
        ((4, 64, 48), -2, False, np.float32, torch.bfloat16),
        ((2, 96, 64), -1, True, np.float32, torch.float32),
        ((2, 96, 64), -1, False, np.float32, torch.bfloat16),
        ((128, 256), -2, True, "bf16", torch.bfloat16),
        ((33, 80), -2, True, np.float32, torch.float32),
    ],
)
def test_quantize_bit_exact(shape, in_axis, per_channel, src_dtype, scale_dtype):
    rng = np.random.default_rng(11)
    w = normal(rng, shape, 0.02)
    if src_dtype == "bf16":
        w = w.astype(O.BF16)
    g = _gpu_q(w, per_channel, in_axis, scale_dtype)
    o = _oracle_q(w.astype(np.float32), per_channel, in_axis, np.float32 if scale_dtype == torch.float32 else O.BF16)
    _same_q(g, o)
    # K-major storage, kappa's logical shape
    assert tuple(g.values.shape) == shape
    assert g.values.stride(in_axis) == 1
    # to_compute_dtype: exact (one rounding per product, as kappa)
    for dt, odt in ((torch.bfloat16, O.BF16), (torch.float32, np.float32)):
        got = to_np(to_compute_dtype(g, dt, in_axis=in_axis)).astype(np.float32)
        ref = O.to_compute_dtype(o, odt).astype(np.float32)
        np.testing.assert_array_equal(got, ref)


# -------------------------------------------------------------- routing ----


def test_topk_known_answers_gpu():
    for case in json.load(open(os.path.join(GOLDEN, "kat_topk.json"))):
        logits = to_dev(np.asarray(case["logits"], dtype=np.float32))
        idx, _ = M.topk_softmax(logits, case["k"])
        np.testing.assert_array_equal(to_np(idx), np.asarray(case["idx"]))


@pytest.mark.parametrize("E,k", [(128, 8), (8, 2), (60, 4), (256, 8)])
def test_topk_exact_on_given_logits(E, k):
    rng = np.random.default_rng(E + k)
    T = 777
    logits = normal(rng, (T, E))
    # plant exact ties, including across the k-th boundary
    logits[::3, 5 % E] = logits[::3, 0]
    logits[::5] = np.round(logits[::5] * 4) / 4
    idx, w = M.topk_softmax(to_dev(logits), k)
    oi, ow = O.topk_softmax(logits, k)
    np.testing.assert_array_equal(to_np(idx), oi)
    # softmax weights: same to within one bf16 rounding step
    np.testing.assert_allclose(to_np(w).astype(np.float32), ow.astype(np.float32), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize(
    "T,k,E,capacity,dist",
    [(1000, 8, 128, None, "uniform"), (513, 2, 8, None, "skewed"), (64, 8, 128, None, "one"),
     (700, 4, 16, 100, "skewed"), (1, 8, 128, None, "uniform"), (4096, 8, 128, None, "uniform"),
     (8192, 8, 256, None, "uniform"), (6000, 4, 64, 300, "skewed")],
)
def test_permute_exact(T, k, E, capacity, dist):
    rng = np.random.default_rng(T * 31 + E)
    if dist == "uniform":
        idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    elif dist == "skewed":
        p = np.arange(1, E + 1, dtype=np.float64) ** 3
        idx = np.stack([rng.choice(E, size=k, replace=False, p=p / p.sum()) for _ in range(T)]).astype(np.int32)
    else:
        idx = np.tile(np.arange(k, dtype=np.int32), (T, 1))
    order, o_sizes, _ = O.permute(idx, E, capacity)
    n = int(o_sizes.sum())
    inv_ref = np.full(T * k, -1, dtype=np.int32)
    inv_ref[order] = np.arange(n, dtype=np.int32)
    for single_block in (False, True):  # kw8_moe_permute_ws (multi-block) and kw8_moe_permute
        st, inv, sizes, offs = M.permute(to_dev(idx), E, capacity, single_block=single_block)
        np.testing.assert_array_equal(to_np(sizes), o_sizes)
        np.testing.assert_array_equal(to_np(offs), np.concatenate([[0], np.cumsum(o_sizes)]))
        np.testing.assert_array_equal(to_np(st)[:n], order // k)
        np.testing.assert_array_equal(to_np(inv), inv_ref)


@pytest.mark.parametrize("T,D,E,k,per_channel", [(300, 256, 16, 4, True), (64, 2048, 128, 8, False), (4096, 2048, 128, 8, True)])
def test_route_end_to_end(T, D, E, k, per_channel):
    rng = np.random.default_rng(T + D)
    x = normal(rng, (1, T, D)).astype(O.BF16)
    router = normal(rng, (D, E), 0.02)
    g = _gpu_q(router, per_channel)
    o = _oracle_q(router, per_channel)
    _same_q(g, o)
    logits, idx, w = M.route_logits(to_dev(x), g, num_experts=E, num_experts_per_tok=k)
    ref_logits = O.router_logits(x.reshape(T, D), o)
    gl = to_np(logits)
    np.testing.assert_allclose(gl, ref_logits, rtol=1e-4, atol=1e-5 * float(np.abs(ref_logits).max()))
    oi, _ = O.topk_softmax(ref_logits, k)
    gi = to_np(idx)
    mism = np.nonzero(np.any(gi != oi, axis=1))[0]
    # every mismatch must sit on a near-tie of the reference logits
    srt = -np.sort(-ref_logits, axis=1)
    for t in mism:
        gap = np.min(np.abs(np.diff(srt[t, : k + 1])))
        assert gap <= 1e-5 * max(1.0, float(np.abs(srt[t]).max())), (t, gap)
    assert len(mism) <= max(1, T // 500), f"{len(mism)} top-k mismatches"
    # with the GPU's own logits the indices are exactly the oracle's top-k
    oi2, ow2 = O.topk_softmax(gl, k)
    np.testing.assert_array_equal(gi, oi2)
    np.testing.assert_allclose(to_np(w).astype(np.float32), ow2.astype(np.float32), rtol=2 ** -7, atol=1e-6)


# ----------------------------------------------------------------- dense ----


def test_dense_golden_fixture():
    z = np.load(os.path.join(GOLDEN, "oracle_small.npz"))
    x = z["ffn_x"].view(O.BF16)
    gt = _gpu_q(z["ffn_gating"], True, -1)
    lw = _gpu_q(z["ffn_linear"], True, -2)
    y = to_np(feed_forward(to_dev(x), gt, lw, transpose_gating_einsum=True))
    # committed kappa-arithmetic (bf16) vectors: sanity bound
    parity(y, z["ffn_y"].view(O.BF16), tol=KAPPA_BF16_TOL)
    ogt = O.quantize_weight(z["ffn_gating"], per_channel_axis=2, scale_dtype=np.float32)
    olw = O.quantize_weight(z["ffn_linear"], per_channel_axis=0, scale_dtype=np.float32)
    parity(y, O.feed_forward(x, ogt, olw, transpose_gating_einsum=True, compute_dtype=np.float32))


@pytest.mark.parametrize("path", [0, 1, 2])
@pytest.mark.parametrize("T,D,H,per_channel", [(200, 256, 512, True), (7, 128, 256, False), (256, 2560, 10240, True),
                                                 (16, 2560, 10240, True), (13, 208, 336, True)])
def test_gemma_feed_forward(path, T, D, H, per_channel):
    if T >= 256 and path == 2:
        pytest.skip("the weight-streaming path is for decode sizes")
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    rng = np.random.default_rng(T + H)
    x = normal(rng, (1, T, D)).astype(O.BF16)
    gating = normal(rng, (2, H, D), 0.02)
    linear = normal(rng, (H, D), 0.02)
    gt, lw = _gpu_q(gating, per_channel, -1), _gpu_q(linear, per_channel, -2)
    ogt, olw = _oracle_q(gating, per_channel, -1), _oracle_q(linear, per_channel, -2)
    _same_q(gt, ogt)
    _same_q(lw, olw)
    y = to_np(feed_forward(to_dev(x), gt, lw, transpose_gating_einsum=True))
    parity(y, O.feed_forward(x, ogt, olw, transpose_gating_einsum=True, compute_dtype=np.float32))
    parity(y, O.feed_forward(x, ogt, olw, transpose_gating_einsum=True), tol=KAPPA_BF16_TOL)


def test_gemma_feed_forward_untransposed_layout():
    rng = np.random.default_rng(5)
    T, D, H = 48, 128, 256
    x = normal(rng, (2, T // 2, D)).astype(O.BF16)
    gating = normal(rng, (2, D, H), 0.02)  # transpose_gating_einsum=False layout
    linear = normal(rng, (H, D), 0.02)
    gt, lw = _gpu_q(gating, True, -2), _gpu_q(linear, True, -2)
    y = feed_forward(to_dev(x), gt, lw, transpose_gating_einsum=False)
    ref = O.feed_forward(x, _oracle_q(gating, True, -2), _oracle_q(linear, True, -2), transpose_gating_einsum=False,
                         compute_dtype=np.float32)
    parity(to_np(y), ref)


@pytest.mark.parametrize("path", [0, 1, 2])
def test_qwen_swiglu_ffn(path):
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    rng = np.random.default_rng(9)
    T, D, I = 40, 256, 384
    x = normal(rng, (1, T, D)).astype(O.BF16)
    ws = [normal(rng, s, 0.02) for s in ((D, I), (D, I), (I, D))]
    g = [_gpu_q(w, False, scale_dtype=torch.bfloat16) for w in ws]  # kappa's per-tensor bf16 scale
    o = [_oracle_q(w, False, scale_dtype=O.BF16) for w in ws]
    y = to_np(swiglu_ffn(to_dev(x), *g))
    parity(y, O.swiglu_ffn(x, *o, compute_dtype=np.float32))
    parity(y, O.swiglu_ffn(x, *o), tol=KAPPA_BF16_TOL)


@pytest.mark.parametrize("T", [7, 100])
def test_qwen3_4b_swiglu_ffn(T):
    """Qwen3-4B dense MLP shape (kappa/qwen3/architecture.py:82-83): D=2560,
    I=9728 (a multiple of 16 but not of 128: the down projection's last k
    stage is partial), kappa's per-tensor bf16 scales."""
    rng = np.random.default_rng(T)
    D, I = 2560, 9728
    x = normal(rng, (1, T, D)).astype(O.BF16)
    ws = [normal(rng, s, 0.02) for s in ((D, I), (D, I), (I, D))]
    g = [_gpu_q(w, False, scale_dtype=torch.bfloat16) for w in ws]
    o = [_oracle_q(w, False, scale_dtype=O.BF16) for w in ws]
    y = to_np(swiglu_ffn(to_dev(x), *g))
    parity(y, O.swiglu_ffn(x, *o, compute_dtype=np.float32))


# ------------------------------------------------------------------- MoE ----


def _moe_check(x, g, o, E, k, y_gpu, capacity=None):
    """Parity of a GPU MoE layer output against the fp32 reference.

    Routing is checked first: top-k sets that differ between the GPU's fp32
    logits and the oracle's must sit on near-ties (gap <= 1e-5 relative
    between the k-th and (k+1)-th reference logit, at most one per 500
    tokens), and where the choice agrees the bf16 routing weights must agree
    to within one bf16 rounding step.  The float comparison then runs the
    reference on the GPU's own routing, so it measures the expert compute
    and the combine over every token.
    """
    T = x.shape[0] * x.shape[1]
    _, gidx, gw = M.route_logits(to_dev(x), g[0], num_experts=E, num_experts_per_tok=k)
    gi, gwn = to_np(gidx), to_np(gw)
    _, oi, ow = O.moe_reference_f32(x, *o, num_experts=E, k=k, capacity=capacity)
    flips = np.nonzero(np.any(np.sort(gi, 1) != np.sort(oi, 1), axis=1))[0]
    if flips.size:
        logits = O.router_logits(x.reshape(T, -1), o[0])
        srt = -np.sort(-logits, axis=1)
        for t in flips:
            gap = float(srt[t, k - 1] - srt[t, k])
            assert gap <= 1e-5 * max(1.0, float(np.abs(srt[t]).max())), f"token {t}: top-k differs, gap {gap}"
        assert flips.size <= max(1, T // 500), f"{flips.size} routing flips"
    same = np.all(gi == oi, axis=1)
    np.testing.assert_allclose(gwn[same].astype(np.float32), ow[same].astype(np.float32), rtol=2 ** -7, atol=1e-6)
    ref, _, _ = O.moe_reference_f32(x, *o, num_experts=E, k=k, capacity=capacity, idx=gi, w=gwn)
    return parity(to_np(y_gpu), ref)


def _moe_case(T, D, I, E, k, per_channel=True, seed=0):
    rng = np.random.default_rng(seed)
    x = normal(rng, (1, T, D)).astype(O.BF16)
    ws = moe_weights(rng, D, I, E)
    g = [_gpu_q(w, per_channel) for w in ws]
    o = [_oracle_q(w, per_channel) for w in ws]
    return x, g, o


def test_moe_golden_fixture():
    z = np.load(os.path.join(GOLDEN, "oracle_small.npz"))
    T, D, I, E, k = (int(v) for v in z["moe_shape"])
    x = z["moe_x"].view(O.BF16)
    g = [_gpu_q(z[n], True) for n in ("moe_router", "moe_gate", "moe_up", "moe_down")]
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    parity(to_np(y), z["moe_y"].view(O.BF16), tol=KAPPA_BF16_TOL)
    o = [O.quantize_weight(z[n], per_channel_axis=z[n].ndim - 2, scale_dtype=np.float32)
         for n in ("moe_router", "moe_gate", "moe_up", "moe_down")]
    _moe_check(x, g, o, E, k, y)


@pytest.mark.parametrize("path", [0, 1, 2])
@pytest.mark.parametrize("T,D,I,E,k,per_channel", [(300, 256, 128, 16, 4, True), (64, 512, 256, 32, 8, False), (5, 256, 128, 16, 4, True),
                                                   (40, 208, 80, 8, 2, True)])
def test_moe_layer_vs_oracle(path, T, D, I, E, k, per_channel):
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    x, g, o = _moe_case(T, D, I, E, k, per_channel, seed=T + E)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    _moe_check(x, g, o, E, k, y)
    # the dispatch kappa would pick (gather_einsum) is the same function; the
    # fused combine adds the k expert rows with fp32 atomics, so two runs
    # agree to fp32 rounding (then bf16), not bit for bit
    y2 = M.moe_swiglu_ffn(to_dev(x), *g, cfg=replace(cfg, moe_impl="gather_einsum"))
    diff = np.abs(to_np(y2).astype(np.float32) - to_np(y).astype(np.float32))
    assert float(diff.max()) <= 2 ** -7 * float(np.abs(to_np(y).astype(np.float32)).max())


@pytest.mark.parametrize("path", [1, 2])
def test_moe_staged_entry_points(path):
    """kw8_moe_route -> kw8_moe_permute -> kw8_moe_expert_ffn -> kw8_moe_combine
    (kappa's _moe_ragged stages, expert outputs stored as bf16 like
    ffn_moe.py:213) against the fused layer."""
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    T, D, I, E, k = 200, 256, 128, 16, 4
    x, g, o = _moe_case(T, D, I, E, k, True, seed=21)
    xd = to_dev(x)
    _, idx, w = M.route_logits(xd, g[0], num_experts=E, num_experts_per_tok=k)
    st, inv, sizes, offs = M.permute(idx, E)
    n = int(to_np(offs)[-1])
    assert n == T * k
    xs = xd.reshape(T, D)[st.long()].contiguous()
    ys = M.expert_ffn(xs, offs, *g[1:])
    y_staged = to_np(M.combine(ys, inv, w, D)).astype(np.float32)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    y_fused = to_np(M.moe_swiglu_ffn(xd, *g, cfg=cfg)).astype(np.float32).reshape(T, D)
    parity(y_staged, y_fused, tol=2e-2)
    ref, _, _ = O.moe_reference_f32(x, *o, num_experts=E, k=k, idx=to_np(idx), w=to_np(w))
    parity(y_staged, ref.reshape(T, D), tol=2e-2)


@pytest.mark.parametrize("T", [256, 24])  # 24 x 2 rows: the one-launch decode routing, 4 of 6 kept
def test_moe_fixed_capacity_vs_oracle(T):
    D, I, E, k = 256, 128, 8, 2
    x, g, o = _moe_case(T, D, I, E, k, True, seed=77)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="fixed_capacity",
                    moe_capacity_factor=0.75, moe_fixed_capacity_slots=1024)
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    _moe_check(x, g, o, E, k, y, capacity=M.fixed_capacity(cfg, T))


def test_moe_token_tiles_agree():
    """Every tensor-core token tile gives the same result (ragged tails, N rounding)."""
    T, D, I, E, k = 500, 256, 192, 16, 4
    x, g, o = _moe_case(T, D, I, E, k, True, seed=3)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    _lib.set_option(_lib.OPT_GEMM_PATH, 1)
    for nt in (16, 48, 128, 192):
        _lib.set_option(_lib.OPT_TOKEN_TILE, nt)
        _moe_check(x, g, o, E, k, M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg))


@pytest.mark.parametrize("nt", [0, 16, 48, 160, 192, 256])
def test_tc_pair_kernel_matches_single_cta(nt):
    """The CTA-pair tensor-core GEMM (M = 256 over two SMs) and the one-CTA
    kernel give the same MoE layer and dense FFN: every epilogue mode, token
    tiles from 32 to 256 (ragged tails, odd group sizes), K not a multiple of
    128, and the split-K dense down projection."""
    _lib.set_option(_lib.OPT_GEMM_PATH, 1)
    _lib.set_option(_lib.OPT_TOKEN_TILE, nt)
    T, D, I, E, k = 700, 208, 336, 16, 4
    x, g, o = _moe_case(T, D, I, E, k, True, seed=nt + 1)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    ys = {}
    for force in (1, 2):
        _lib.set_option(_lib.OPT_TC_PAIR, force)
        ys[force] = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
        _moe_check(x, g, o, E, k, ys[force])
    parity(to_np(ys[2]), to_np(ys[1]), tol=2e-2)
    # dense: gate/up pair mode, plain bf16 down, and the split-K fp32 down
    rng = np.random.default_rng(nt)
    for Tn, Dn, Hn in ((96, 512, 2048), (40, 2560, 10240)):
        xd = normal(rng, (1, Tn, Dn)).astype(O.BF16)
        gating, linear = normal(rng, (2, Hn, Dn), 0.02), normal(rng, (Hn, Dn), 0.02)
        gt, lw = _gpu_q(gating, True, -1), _gpu_q(linear, True, -2)
        ref = O.feed_forward(xd, _oracle_q(gating, True, -1), _oracle_q(linear, True, -2),
                             transpose_gating_einsum=True, compute_dtype=np.float32)
        for force in (1, 2):
            _lib.set_option(_lib.OPT_TC_PAIR, force)
            parity(to_np(feed_forward(to_dev(xd), gt, lw, transpose_gating_einsum=True)), ref)


_FULL = {}


def _full_moe_weights():
    """Qwen3-30B-A3B-shaped W8 weights, seed 0, generated once per session."""
    if not _FULL:
        D, I, E = 2048, 768, 128
        rng = np.random.default_rng(0)
        ws = moe_weights(rng, D, I, E)
        _FULL["g"] = [_gpu_q(w, True) for w in ws]
        _FULL["o"] = [_oracle_q(w, True) for w in ws]
    return _FULL["g"], _FULL["o"]


def test_moe_qwen3_30b_a3b_prefill_vs_oracle():
    """Qwen3-30B-A3B-shaped layer, T=4096, per-channel W8."""
    T, D, E, k = 4096, 2048, 128, 8
    g, o = _full_moe_weights()
    x = normal(np.random.default_rng(100), (1, T, D)).astype(O.BF16)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax")
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    _moe_check(x, g, o, E, k, y)


@pytest.mark.parametrize("B", [1, 8, 64, 256])
def test_moe_qwen3_30b_a3b_decode_vs_oracle(B):
    """decode batches of the same layer."""
    D, E, k = 2048, 128, 8
    g, o = _full_moe_weights()
    x = normal(np.random.default_rng(B), (B, 1, D)).astype(O.BF16)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax")
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    _moe_check(x, g, o, E, k, y)


@pytest.mark.parametrize("T", [5, 300])  # 5 x 4 rows: the one-launch decode routing; 300: the multi-block sort
def test_moe_nan_token_is_reported_and_dropped(T):
    """A token whose router logits are NaN has no top-k order: its expert ids
    are invalid, the device status says KW8_ERR_INVALID_ARG, its output row is
    zero, and every other token gets the result it gets without it."""
    D, I, E, k = 256, 128, 16, 4
    x, g, _ = _moe_case(T, D, I, E, k, True, seed=91)
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax",
                    moe_ragged_decode_token_threshold=0)
    xd = to_dev(x)
    xd[0, 0] = float("nan")
    assert _lib.device_status(xd) == 0
    y = M.moe_swiglu_ffn(xd, *g, cfg=cfg).float()
    assert _lib.device_status(xd) == _lib.KW8_ERR_INVALID_ARG
    assert float(y[0, 0].abs().max()) == 0.0
    rest = M.moe_swiglu_ffn(xd[:, 1:].contiguous(), *g, cfg=cfg).float()
    assert _lib.device_status(xd) == 0
    assert float((y[0, 1:] - rest[0]).abs().max()) <= 2 ** -7 * float(rest.abs().max())


def test_moe_errors_match_kappa():
    T, D, I, E, k = 8, 64, 32, 4, 2
    x, g, _ = _moe_case(T, D, I, E, k)
    with pytest.raises(ValueError, match="use_moe"):
        M.moe_swiglu_ffn(to_dev(x), *g, cfg=MoEConfig(use_moe=False, num_experts=E, num_experts_per_tok=k))
    with pytest.raises(ValueError, match="unknown moe_impl"):
        M.moe_swiglu_ffn(to_dev(x), *g, cfg=MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="nope"))
    with pytest.raises(ValueError, match="router_w shape"):
        M.moe_swiglu_ffn(to_dev(x), *g, cfg=MoEConfig(use_moe=True, num_experts=E + 1, num_experts_per_tok=k))
    with pytest.raises(ValueError, match="moe_capacity_factor"):
        M.moe_swiglu_ffn(to_dev(x), *g, cfg=MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k,
                                                      moe_impl="fixed_capacity", moe_capacity_factor=0.0))


def _ep_single_rank_peers(dev, Tm, D, E, k, dedup, ret_format=_lib.RET_F16_SCALED, red_rows=0):
    """A one-rank expert-parallel group: its own buffers are the peers'."""
    world = 1
    bufs = {
        "recv": torch.zeros((world * Tm * k, D), dtype=torch.bfloat16, device=dev),
        "out": torch.zeros((Tm * k, D), dtype=torch.bfloat16, device=dev),
        "counts": torch.zeros(2 * world * (E + world), dtype=torch.int32, device=dev),
        "flags": torch.zeros(3 * world + 3, dtype=torch.int32, device=dev),
        "rows": torch.zeros((world * Tm, D), dtype=torch.bfloat16, device=dev),
        "meta": torch.zeros(2 * world * Tm * k, dtype=torch.int32, device=dev),
        # rows of D partial sums (4 or 2 bytes each) + one fp32 scale per row (fp16 rows)
        "ret": torch.zeros(world * Tm * (D * (4 if ret_format == _lib.RET_F32 else 2) + 4), dtype=torch.uint8,
                           device=dev),
        "red": torch.zeros((2, world, max(red_rows, 1), D), dtype=torch.float32, device=dev),
    }
    arr = {n: torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev) for n, t in bufs.items()}
    p = _lib.KW8EpPeers(
        world, 0, Tm, arr["recv"].data_ptr(), arr["out"].data_ptr(), arr["counts"].data_ptr(),
        arr["flags"].data_ptr(), bufs["recv"].data_ptr(), bufs["out"].data_ptr(), bufs["counts"].data_ptr(),
        bufs["flags"].data_ptr(),
        arr["rows"].data_ptr() if dedup else None, arr["meta"].data_ptr() if dedup else None,
        arr["ret"].data_ptr() if dedup else None, bufs["rows"].data_ptr() if dedup else None,
        bufs["meta"].data_ptr() if dedup else None, bufs["ret"].data_ptr() if dedup else None, ret_format,
        arr["red"].data_ptr(), bufs["red"].data_ptr(), red_rows)
    return p, (bufs, arr)


@pytest.mark.parametrize("dedup,ret_format", [(True, _lib.RET_F16_SCALED), (True, _lib.RET_F32), (True, _lib.RET_BF16),
                                               (False, _lib.RET_F16_SCALED)])
def test_moe_ep_single_rank(dedup, ret_format):
    """kw8_moe_ffn_ep on a group of one rank: every step of the expert-parallel
    call (counts exchange, row and record dispatch, phase flags, local
    experts, return, combine) runs on one GPU against the fp32 reference, for
    two calls in a row (epochs 1 and 2, both count copies).  The partial sums
    return as fp16 with a per-row scale, fp32 or bf16."""
    import ctypes

    from kappa_b200.qwen3.quant import kmajor

    T, D, I, E, k = 200, 256, 128, 16, 4
    x, g, o = _moe_case(T, D, I, E, k, True, seed=31)
    dev = torch.device("cuda", 0)
    peers, keep = _ep_single_rank_peers(dev, T, D, E, k, dedup, ret_format)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_moe_ffn_ep_workspace_size(T, D, I, E, k, 1)), dtype=torch.uint8, device=dev)
    km = [kmajor(w, -2) for w in g]
    xd = to_dev(x).reshape(T, D)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.set_option(_lib.OPT_EP_TIMING, 1 if dedup else 0)
    try:
        for epoch in (1, 2):
            out = torch.empty_like(xd)
            _lib.check(lib.kw8_moe_ffn_ep(xd.data_ptr(), T, D, I, E, k, -1, *[w.struct() for w in km],
                                          out.data_ptr(), ctypes.byref(peers), epoch, ws.data_ptr(), ws.numel(),
                                          stream))
            assert _lib.device_status(out) == 0
            _moe_check(x, g, o, E, k, out.reshape(1, T, D))
        if dedup:  # the phase times of the last call (CUDA events at its phase boundaries)
            ms = (ctypes.c_float * 9)()
            _lib.check(lib.kw8_ep_phase_times(ms, 9))
            assert all(v >= 0.0 for v in ms) and sum(ms) > 0.0
    finally:
        _lib.set_option(_lib.OPT_EP_TIMING, 0)
    del keep


@pytest.mark.parametrize("B", [1, 8, 64, 256])
def test_moe_ep_decode_single_rank(B):
    """kw8_moe_ffn_ep_decode on a group of one rank: routing of the
    replicated batch, the local experts' fused combine, the push of the fp32
    partial into the exchange slot, the flag phase and the rank-order sum, for
    three calls in a row (both slot parities), against the fp32 reference."""
    import ctypes

    from kappa_b200.qwen3.quant import kmajor

    D, I, E, k = 512, 256, 32, 8
    x, g, o = _moe_case(B, D, I, E, k, True, seed=B + 5)
    dev = torch.device("cuda", 0)
    peers, keep = _ep_single_rank_peers(dev, B, D, E, k, True, red_rows=256)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_moe_ffn_ep_decode_workspace_size(B, D, I, E, k)), dtype=torch.uint8, device=dev)
    km = [kmajor(w, -2) for w in g]
    xd = to_dev(x).reshape(B, D)
    stream = torch.cuda.current_stream(dev).cuda_stream
    outs = []
    for epoch in (1, 2, 3):
        out = torch.empty_like(xd)
        _lib.check(lib.kw8_moe_ffn_ep_decode(xd.data_ptr(), B, D, I, E, k, -1, *[w.struct() for w in km],
                                             out.data_ptr(), ctypes.byref(peers), epoch, ws.data_ptr(), ws.numel(),
                                             stream))
        assert _lib.device_status(out) == 0
        _moe_check(x, g, o, E, k, out.reshape(1, B, D))
        outs.append(out)
    del keep


@pytest.mark.parametrize("T,act", [(16, 0), (300, 1)])
def test_dense_ffn_tp_single_rank(T, act):
    """kw8_dense_ffn_tp on a group of one rank (the whole hidden axis is the
    rank's shard): the fp32 partial's push, flag phase and sum equal the
    dense FFN."""
    import ctypes

    from kappa_b200.qwen3.quant import kmajor

    D, H = 512, 1024
    rng = np.random.default_rng(T)
    x = normal(rng, (1, T, D)).astype(O.BF16)
    gating, linear = normal(rng, (2, H, D), 0.02), normal(rng, (H, D), 0.02)
    gt, lw = _gpu_q(gating, True, -1), _gpu_q(linear, True, -2)
    dev = torch.device("cuda", 0)
    peers, keep = _ep_single_rank_peers(dev, 1, D, 4, 1, False, red_rows=512)
    g, l2 = kmajor(gt, -1), kmajor(lw, -2)
    lib = _lib.load()
    ws = torch.empty(int(lib.kw8_dense_ffn_tp_workspace_size(T, D, H)), dtype=torch.uint8, device=dev)
    xd = to_dev(x).reshape(T, D)
    out = torch.empty_like(xd)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.kw8_dense_ffn_tp(xd.data_ptr(), T, D, H, g.struct(0), g.struct(H), l2.struct(), act,
                                    out.data_ptr(), ctypes.byref(peers), 1, ws.data_ptr(), ws.numel(), stream))
    assert _lib.device_status(out) == 0
    # epoch 0: the group's device-side call count (word 3 * world of the
    # flags), three eager calls and then the call captured in a CUDA graph
    # and replayed twice: each call takes the next tag and the same result.
    keep[0]["flags"].zero_()
    outs = []
    for _ in range(3):
        o = torch.empty_like(xd)
        _lib.check(lib.kw8_dense_ffn_tp(xd.data_ptr(), T, D, H, g.struct(0), g.struct(H), l2.struct(), act,
                                        o.data_ptr(), ctypes.byref(peers), 0, ws.data_ptr(), ws.numel(), stream))
        outs.append(o)
    assert _lib.device_status(out) == 0
    assert int(keep[0]["flags"][3].item()) == 3
    graph_out = torch.empty_like(xd)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        _lib.check(lib.kw8_dense_ffn_tp(xd.data_ptr(), T, D, H, g.struct(0), g.struct(H), l2.struct(), act,
                                        graph_out.data_ptr(), ctypes.byref(peers), 0, ws.data_ptr(), ws.numel(),
                                        side.cuda_stream))
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)
    assert int(keep[0]["flags"][3].item()) == 5
    for o in outs + [graph_out]:
        assert torch.equal(o, out)
    del graph
    assert _lib.device_status(out) == 0
    ogt, olw = _oracle_q(gating, True, -1), _oracle_q(linear, True, -2)
    if act == 0:
        ref = O.feed_forward(x, ogt, olw, transpose_gating_einsum=True, compute_dtype=np.float32)
    else:
        ref = O.swiglu_ffn(x, O.Q8Weight(np.swapaxes(ogt.values[0], 0, 1), np.swapaxes(ogt.scale[0], 0, 1)),
                           O.Q8Weight(np.swapaxes(ogt.values[1], 0, 1), np.swapaxes(ogt.scale[1], 0, 1)), olw,
                           compute_dtype=np.float32)
    parity(to_np(out).reshape(1, T, D), ref)
    del keep


def test_ep_barrier_wait_times_out():
    """Failure detection of the expert-parallel phase flags without a fault:
    a wait for a phase that no rank marks runs out after its bound (about
    2 s), records KW8_ERR_DEVICE_TIMEOUT in the device status and returns;
    the context stays usable and a signalled phase then passes."""
    import ctypes

    dev = torch.device("cuda", 0)
    counts = torch.zeros(2 * 1 * 8, dtype=torch.int32, device=dev)
    flags = torch.zeros(3, dtype=torch.int32, device=dev)
    buf = torch.zeros(64, dtype=torch.uint8, device=dev)
    arr = [torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev) for t in (buf, buf, counts, flags)]
    peers = _lib.KW8EpPeers(1, 0, 0, arr[0].data_ptr(), arr[1].data_ptr(), arr[2].data_ptr(), arr[3].data_ptr(),
                            buf.data_ptr(), buf.data_ptr(), counts.data_ptr(), flags.data_ptr())
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.kw8_ep_barrier(ctypes.byref(peers), 1, 7, 0, stream))  # nobody marks epoch 7
    assert _lib.device_status(buf) == _lib.KW8_ERR_DEVICE_TIMEOUT
    _lib.check(lib.kw8_ep_barrier(ctypes.byref(peers), 1, 7, 1, stream))  # this rank marks it
    assert _lib.device_status(buf) == 0
    assert int(flags[1].item()) == 7
