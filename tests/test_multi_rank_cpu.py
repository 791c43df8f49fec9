"""Multi-rank host logic on CPU: gloo, world size 2, spawned ranks.

The exchange code of kappa_b200.qwen3.sharding (expert-parallel MoE, tensor
parallel dense MLP) runs unchanged; its compute steps are supplied by the
NumPy oracle (OracleMoEOps), which is test infrastructure only.  Checks:

* EP prefill / decode: each rank's output matches the same ops run on that
  rank's tokens with every expert (no exchange; BLAS may order a row's sums
  differently for another batch size, hence a 1e-3 bar rather than bit
  equality), and the fp32 dequantise-then-dot reference within the parity
  bar;
* TP: the shard helpers (scales split with output channels, replicated
  otherwise) plus one all-reduce reproduce the full dense MLP;
* regroup_index against a direct construction.
"""

from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from oracle import kappa_ref as KR
from helpers import moe_weights, normal, parity, to_np

WORLD = 2


def _t(a: np.ndarray) -> torch.Tensor:
    """numpy (bf16 or other) -> CPU torch tensor."""
    a = np.ascontiguousarray(a)
    if a.dtype == O.BF16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


class OracleMoEOps:
    """MoEOps on CPU tensors with the oracle's arithmetic (fp32 expert compute)."""

    def __init__(self, k: int):
        self.k = k

    def route(self, x_flat, router_w, num_experts, k):
        logits = O.router_logits(to_np(x_flat), router_w)
        idx, w = O.topk_softmax(logits, k, out_dtype=O.BF16)
        return _t(idx.astype(np.int32)), _t(w)

    def permute(self, idx, num_experts, capacity):
        k = idx.shape[1]
        order, sizes, _ = O.permute(to_np(idx), num_experts, capacity)
        m = idx.numel()
        inv = np.full(m, -1, dtype=np.int32)
        inv[order] = np.arange(order.size, dtype=np.int32)
        sorted_token = np.full(m, -1, dtype=np.int32)
        sorted_token[: order.size] = (order // k).astype(np.int32)
        offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
        return _t(sorted_token), _t(inv), _t(sizes.astype(np.int32)), _t(offsets)

    def gather(self, x_flat, sorted_token, rows):
        return x_flat.index_select(0, sorted_token[:rows].long())

    def experts(self, xs, group_offsets, gate, up, down):
        xf = to_np(xs).astype(np.float32)
        sizes = np.diff(to_np(group_offsets).astype(np.int64))
        g = KR._ragged_dot(xf, O.to_compute_dtype(gate, np.float32), sizes)
        u = KR._ragged_dot(xf, O.to_compute_dtype(up, np.float32), sizes)
        h = (KR.silu(g) * u).astype(np.float32)
        y = KR._ragged_dot(h, O.to_compute_dtype(down, np.float32), sizes)
        return _t(y.astype(O.BF16))

    def combine(self, ys, inv_pos, w, d):
        yf = to_np(ys).astype(np.float32)
        inv = to_np(inv_pos)
        wf = to_np(w).astype(np.float32)
        T, k = wf.shape
        out = np.zeros((T, d), dtype=np.float32)
        for j in range(k):
            p = inv.reshape(T, k)[:, j]
            keep = p >= 0
            out[keep] += wf[keep, j : j + 1] * yf[p[keep]]
        return _t(out.astype(O.BF16))


class _Cfg:
    use_moe = True
    moe_impl = "ragged_jax"
    moe_capacity_factor = 1.25
    moe_fixed_capacity_slots = None
    moe_ragged_decode_token_threshold = 64

    def __init__(self, e, k):
        self.num_experts = e
        self.num_experts_per_tok = k


def _local_all_experts(ops, x, router, gate, up, down, e, k):
    """The same ops on one rank's tokens with every expert, no exchange."""
    b, t, d = x.shape
    x_flat = x.reshape(b * t, d)
    idx, w = ops.route(x_flat, router, e, k)
    st, inv, sizes, offs = ops.permute(idx, e, None)
    kept = int(offs[e])
    ys = ops.experts(ops.gather(x_flat, st, kept), offs, gate, up, down)
    return ops.combine(ys, inv, w, d).reshape(b, t, d)


def _slice_q8(w: O.Q8Weight, sl: slice) -> O.Q8Weight:
    scale = w.scale[sl] if np.ndim(w.scale) == w.values.ndim else w.scale
    return O.Q8Weight(values=w.values[sl], scale=scale)


def _rank_main(rank: int, world: int, port: int, errfile: str):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from kappa_b200.qwen3 import sharding as S
        from kappa_b200.qwen3.quant import Q8Weight as TQ8

        # ---------------------------------------------------- MoE, EP ----
        D, I, E, K = 64, 32, 8, 2
        rng = np.random.default_rng(0)  # identical weights on every rank
        r, g, u, dn = moe_weights(rng, D, I, E)
        router = O.quantize_weight(r, per_channel_axis=-2, scale_dtype=np.float32)
        gate = O.quantize_weight(g, per_channel_axis=-2, scale_dtype=np.float32)
        up = O.quantize_weight(u, per_channel_axis=-2, scale_dtype=np.float32)
        down = O.quantize_weight(dn, per_channel_axis=-2, scale_dtype=np.float32)
        e_loc = E // world
        sl = slice(rank * e_loc, (rank + 1) * e_loc)
        gl, ul, dl = _slice_q8(gate, sl), _slice_q8(up, sl), _slice_q8(down, sl)
        ops = OracleMoEOps(K)
        cfg = _Cfg(E, K)
        xr = np.random.default_rng(100 + rank)  # each rank's own tokens (uneven routing per rank)
        x = normal(xr, (1, 24 + 8 * rank, D)).astype(O.BF16)
        xt = _t(x)
        y_ep = S.moe_swiglu_ffn_ep(xt, router, gl, ul, dl, cfg=cfg, ops=ops)
        y_loc = _local_all_experts(ops, xt, router, gate, up, down, E, K)
        parity(to_np(y_ep), to_np(y_loc), tol=1e-3)
        ref, _, _ = O.moe_reference_f32(x, router, gate, up, down, num_experts=E, k=K)
        parity(to_np(y_ep), ref)

        # decode: replicated x, local experts, one all-reduce
        xd = normal(np.random.default_rng(7), (1, 4, D)).astype(O.BF16)
        y_dec = S.moe_swiglu_ffn_ep_decode(_t(xd), router, gl, ul, dl, cfg=cfg, ops=ops)
        ref_d, _, _ = O.moe_reference_f32(xd, router, gate, up, down, num_experts=E, k=K)
        parity(to_np(y_dec), ref_d)

        # ------------------------------------------------ dense MLP, TP ----
        Dd, H = 32, 48
        rng2 = np.random.default_rng(3)
        gw = O.quantize_weight(normal(rng2, (Dd, H), 0.05), per_channel_axis=-2, scale_dtype=np.float32)
        uw = O.quantize_weight(normal(rng2, (Dd, H), 0.05), per_channel_axis=-2, scale_dtype=np.float32)
        dw = O.quantize_weight(normal(rng2, (H, Dd), 0.05), per_channel_axis=-2, scale_dtype=np.float32)
        xm = normal(np.random.default_rng(11), (1, 5, Dd)).astype(O.BF16)

        def tq(w: O.Q8Weight) -> TQ8:
            return TQ8(values=torch.from_numpy(w.values.copy()), scale=torch.from_numpy(np.asarray(w.scale).copy()))

        def oq(w: TQ8) -> O.Q8Weight:
            return O.Q8Weight(values=w.values.numpy(), scale=w.scale.numpy())

        gs, us, ds = S.shard_dense_swiglu(tq(gw), tq(uw), tq(dw), rank, world)
        assert tuple(gs.values.shape) == (Dd, H // world) and tuple(gs.scale.shape) == (1, H // world)
        assert tuple(ds.values.shape) == (H // world, Dd) and tuple(ds.scale.shape) == (1, Dd)
        part = O.swiglu_ffn(xm, oq(gs), oq(us), oq(ds), compute_dtype=np.float32)
        pt = torch.from_numpy(np.ascontiguousarray(part, dtype=np.float32))
        dist.all_reduce(pt)
        full = O.swiglu_ffn(xm, gw, uw, dw, compute_dtype=np.float32)
        np.testing.assert_allclose(pt.numpy(), full, rtol=1e-4, atol=1e-4 * float(np.abs(full).max()))

        # Gemma gating [2, H, D] (transposed einsum) split on H, linear [H, D] split on H
        gg = O.quantize_weight(normal(rng2, (2, H, Dd), 0.05), per_channel_axis=-1, scale_dtype=np.float32)
        ll = O.quantize_weight(normal(rng2, (H, Dd), 0.05), per_channel_axis=-2, scale_dtype=np.float32)
        gsh, lsh = S.shard_gemma_mlp(tq(gg), tq(ll), rank, world, transpose_gating_einsum=True)
        assert tuple(gsh.values.shape) == (2, H // world, Dd) and tuple(gsh.scale.shape) == (2, H // world, 1)
        part = O.feed_forward(xm, oq(gsh), oq(lsh), transpose_gating_einsum=True, compute_dtype=np.float32)
        pt = torch.from_numpy(np.ascontiguousarray(part, dtype=np.float32))
        dist.all_reduce(pt)
        full = O.feed_forward(xm, gg, ll, transpose_gating_einsum=True, compute_dtype=np.float32)
        np.testing.assert_allclose(pt.numpy(), full, rtol=1e-4, atol=1e-4 * float(np.abs(full).max()))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # reported to the parent through the file
        with open(errfile, "a") as f:
            f.write(f"rank {rank}: {type(exc).__name__}: {exc}\n")
        raise


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_tp_two_ranks_gloo():
    with tempfile.NamedTemporaryFile("w+", suffix=".log", delete=False) as f:
        errfile = f.name
    try:
        mp.start_processes(_rank_main, args=(WORLD, _free_port(), errfile), nprocs=WORLD, start_method="spawn")
    except Exception:
        with open(errfile) as f:
            pytest.fail(f.read() or "a rank failed")
    finally:
        os.unlink(errfile)


def test_regroup_index():
    from kappa_b200.qwen3.sharding import regroup_index

    counts = torch.tensor([[2, 0, 3], [1, 4, 0], [0, 2, 1]])
    world, e_loc = counts.shape
    rows = []  # source-major labels (s, j, r)
    for s in range(world):
        for j in range(e_loc):
            rows += [(s, j, r) for r in range(int(counts[s, j]))]
    want = sorted(range(len(rows)), key=lambda i: (rows[i][1], rows[i][0], rows[i][2]))
    assert regroup_index(counts).tolist() == want
    assert regroup_index(torch.zeros((2, 3), dtype=torch.int64)).numel() == 0
