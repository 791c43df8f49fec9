"""Pre-packed ("tiled") W8 weights on the GPU, through the C ABI.

The packed layout holds the same int8 values in another order, and every
kernel computes the same products in the same order from it, so results are
bit-identical to those from K-major weights (the MoE layers are compared with
the fixed-order combine, whose additions do not depend on timing)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from helpers import moe_weights, normal, parity, to_dev, to_np
from kappa_b200 import _lib
from kappa_b200.gemma3.ffn import feed_forward
from kappa_b200.qwen3 import ffn_moe as M
from kappa_b200.qwen3 import linear as qlin
from kappa_b200.qwen3 import transformer as QT
from kappa_b200.qwen3.architecture import MoEConfig
from kappa_b200.qwen3.ffn import swiglu_ffn
from kappa_b200.qwen3.quant import Q8Tiled, pack_weight, quantize_weight, to_compute_dtype, unpack_weight

pytestmark = pytest.mark.gpu

_OPTS = (_lib.OPT_GEMM_PATH, _lib.OPT_TOKEN_TILE, _lib.OPT_DETERMINISTIC, _lib.OPT_TC_PAIR)


@pytest.fixture(autouse=True)
def _reset_options():
    for opt in _OPTS:
        _lib.set_option(opt, 0)
    yield
    for opt in _OPTS:
        _lib.set_option(opt, 0)
    assert _lib.device_status(torch.zeros(1, device="cuda")) == 0, "a kernel reported a device-side error"


def _np_pack(q: np.ndarray) -> np.ndarray:
    """The tiled layout of include/kappa_w8.h (KW8_LAYOUT_TILED), stated in NumPy:
    [groups][ceil(N/16)][2*ceil(K/128)][1024], row 16f + 8h + r and the 16 k of
    chunk c of step s at byte 512 h + 16 (8 c + r); zeros past N and K."""
    *lead, N, K = q.shape
    g = int(np.prod(lead)) if lead else 1
    FT, KS = -(-N // 16), -(-K // 128) * 2
    pad = np.zeros((g, FT * 16, KS * 64), dtype=np.int8)
    pad[:, :N, :K] = q.reshape(g, N, K)
    # [g][f][h][r][s][c][b] -> [g][f][s][h][c][r][b]
    t = pad.reshape(g, FT, 2, 8, KS, 4, 16).transpose(0, 1, 4, 2, 5, 3, 6)
    return np.ascontiguousarray(t).reshape(g, FT, KS, 1024).view(np.uint8)


@pytest.mark.parametrize("shape,in_axis", [((3, 40, 208), -1), ((2, 256, 100), -2), ((16, 2048), -1),
                                           ((5, 768, 2048), -2), ((48, 80), -2)])
def test_pack_layout_and_round_trip(shape, in_axis):
    rng = np.random.default_rng(sum(shape))
    w = normal(rng, shape, 0.02)
    q = quantize_weight(to_dev(w), per_channel=True, in_axis=in_axis, scale_dtype=torch.float32)
    t = pack_weight(q, in_axis=in_axis)
    assert isinstance(t, Q8Tiled)
    kmaj = q.values.transpose(-1, -2) if in_axis == -2 else q.values
    np.testing.assert_array_equal(to_np(t.tiled), _np_pack(to_np(kmaj.contiguous())))
    back = unpack_weight(t)
    np.testing.assert_array_equal(to_np(back.values), to_np(q.values))
    for dt in (torch.bfloat16, torch.float32):
        assert torch.equal(to_compute_dtype(t, dt, in_axis=in_axis), to_compute_dtype(q, dt, in_axis=in_axis))


@pytest.mark.parametrize("path", [0, 1, 2])
@pytest.mark.parametrize("T,D,H", [(1, 2560, 10240), (7, 208, 336), (16, 512, 1024), (40, 2560, 10240),
                                    (256, 2560, 10240)])
def test_dense_packed_is_bit_identical(path, T, D, H):
    if path == 2 and T > 64:
        pytest.skip("the weight-streaming path is for decode sizes")
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    rng = np.random.default_rng(T + D)
    x = to_dev(normal(rng, (1, T, D)).astype(O.BF16))
    gating = quantize_weight(to_dev(normal(rng, (2, H, D), 0.02)), per_channel=True, in_axis=-1,
                             scale_dtype=torch.float32)
    linear = quantize_weight(to_dev(normal(rng, (H, D), 0.02)), per_channel=True, scale_dtype=torch.float32)
    y = feed_forward(x, gating, linear, transpose_gating_einsum=True)
    yt = feed_forward(x, pack_weight(gating, in_axis=-1), pack_weight(linear), transpose_gating_einsum=True)
    assert torch.equal(y, yt)
    # Qwen3 dense (kappa's per-tensor bf16 scales, [D, I] layouts)
    ws = [quantize_weight(to_dev(normal(rng, s, 0.02)), scale_dtype=torch.bfloat16) for s in ((D, H), (D, H), (H, D))]
    assert torch.equal(swiglu_ffn(x, *ws), swiglu_ffn(x, *[pack_weight(w) for w in ws]))


@pytest.mark.parametrize("path", [0, 1, 2])
@pytest.mark.parametrize("T,D,I,E,k", [(1, 2048, 768, 128, 8), (8, 2048, 768, 128, 8), (64, 2048, 768, 128, 8),
                                        (300, 208, 80, 16, 4), (256, 2048, 768, 128, 8)])
def test_moe_packed_is_bit_identical(path, T, D, I, E, k):
    if path == 2 and T > 64:
        pytest.skip("the weight-streaming path is for decode sizes")
    _lib.set_option(_lib.OPT_GEMM_PATH, path)
    _lib.set_option(_lib.OPT_DETERMINISTIC, 1)
    rng = np.random.default_rng(T + E)
    x = normal(rng, (1, T, D)).astype(O.BF16)
    ws = moe_weights(rng, D, I, E)
    g = [quantize_weight(to_dev(w), per_channel=True, scale_dtype=torch.float32) for w in ws]
    gt = [pack_weight(w) for w in g]
    cfg = MoEConfig(use_moe=True, num_experts=E, num_experts_per_tok=k, moe_impl="ragged_jax")
    y = M.moe_swiglu_ffn(to_dev(x), *g, cfg=cfg)
    yt = M.moe_swiglu_ffn(to_dev(x), *gt, cfg=cfg)
    assert torch.equal(y, yt)
    # and the default fused combine on packed weights meets the parity bar
    _lib.set_option(_lib.OPT_DETERMINISTIC, 0)
    o = [O.quantize_weight(w, per_channel_axis=w.ndim - 2, scale_dtype=np.float32) for w in ws]
    _, idx, wr = M.route_logits(to_dev(x), g[0], num_experts=E, num_experts_per_tok=k)
    ref, _, _ = O.moe_reference_f32(x, *o, num_experts=E, k=k, idx=to_np(idx), w=to_np(wr))
    parity(to_np(M.moe_swiglu_ffn(to_dev(x), *gt, cfg=cfg)), ref)


@pytest.mark.parametrize("T", [1, 5, 200])
def test_linears_packed_are_bit_identical(T):
    rng = np.random.default_rng(T)
    D, nq, hd, V = 2048, 16, 128, 4096
    x = to_dev(normal(rng, (2, T, D)).astype(O.BF16))
    qw = quantize_weight(to_dev(normal(rng, (nq, D, hd), 0.02)), per_channel=True, scale_dtype=torch.float32)
    assert torch.equal(qlin.project_q(x, qw), qlin.project_q(x, pack_weight(qw)))
    head = quantize_weight(to_dev(normal(rng, (V, D), 0.02)), per_channel=True, in_axis=-1, scale_dtype=torch.float32)
    assert torch.equal(QT.logits_from_hidden(x, head), QT.logits_from_hidden(x, pack_weight(head, in_axis=-1)))
