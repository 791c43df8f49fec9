"""Multi-GPU W8 FFN: tensor parallel dense MLP and expert parallel MoE.

One process per GPU, ``torch.distributed`` (NCCL) for the exchanges; every
rank runs the single-GPU kernels on its shard.

Dense MLP (kappa/qwen3/sharding.py:127-132, GSPMD there): gate/up (Gemma's
gating) split on the hidden axis H (column parallel), down (Gemma's linear)
split on H (row parallel).  Per-channel scales follow their output channels:
gate/up scales are split with H, down scales (per model-dim channel) are
replicated, a per-tensor scale is replicated (sharding.py:109-112).  Each
rank computes its fp32 partial of the layer output; one all-reduce (fp32,
so the sum is not rounded per rank) and one cast give the bf16 output.

MoE, expert parallel (not in kappa): rank r holds experts
[r*E/R, (r+1)*E/R) and its own tokens; the router is replicated.
* prefill (``moe_swiglu_ffn_ep``): route and stably sort the rank's routed
  rows by expert, all-gather the per-expert counts, and move every routed
  row of x straight into its expert owner's receive buffer over NVLink
  (``kw8_ep_dispatch``: peer-to-peer stores into CUDA-IPC-mapped buffers
  held by an :class:`EPContext`, laid out expert-major, so the grouped
  expert FFN runs on it directly); the outputs go back the same way
  (``kw8_ep_return``) and each rank combines locally.  Every placement is
  computed on the GPU from the counts: no host round trip.  Two one-element
  all-reduces order the phases across ranks.  Without a context (or with
  custom ``ops``) the rows move with NCCL all-to-allv instead (counts to the
  host, regroup by local expert).  Each rank's result equals the single-GPU
  layer on that rank's tokens.
* decode (``moe_swiglu_ffn_ep_decode``): x is replicated (B x D is small);
  every rank routes all tokens, runs only its local experts' rows and adds
  their weighted outputs into an fp32 partial; one all-reduce sums them.

The compute steps go through an ``ops`` object (default: the B200 kernels),
so the exchange logic also runs on CPU ranks (gloo) in the tests.
"""

from __future__ import annotations

import ctypes
from typing import Protocol

import torch
import torch.distributed as dist

from kappa_b200 import _lib
from kappa_b200.qwen3.quant import Q8Weight, Weight, kmajor

__all__ = [
    "shard_output_channels",
    "shard_input_channels",
    "shard_dense_swiglu",
    "shard_gemma_mlp",
    "shard_experts",
    "swiglu_ffn_tp",
    "feed_forward_tp",
    "moe_swiglu_ffn_ep",
    "EPContext",
    "TPContext",
    "moe_swiglu_ffn_ep_decode",
    "MoEOps",
    "KernelMoEOps",
    "regroup_index",
]


def _world(group) -> tuple[int, int]:
    return dist.get_world_size(group), dist.get_rank(group)


def _span(n: int, rank: int, world: int, what: str) -> slice:
    if n % world:
        raise ValueError(f"{what}={n} is not divisible by the {world} ranks")
    c = n // world
    return slice(rank * c, (rank + 1) * c)


def _q8(w: Weight, name: str) -> Q8Weight:
    if not isinstance(w, Q8Weight):
        raise TypeError(f"{name}: expected a Q8Weight")
    return w


def shard_output_channels(w: Weight, rank: int, world: int, axis: int) -> Q8Weight:
    """Column-parallel shard: output axis ``axis`` split, per-channel scales with it."""
    q = _q8(w, "weight")
    v = q.values
    ax = axis % v.dim()
    sl = [slice(None)] * v.dim()
    sl[ax] = _span(int(v.shape[ax]), rank, world, "output channels")
    values = v[tuple(sl)]
    scale = q.scale
    if scale.dim() == v.dim() and int(scale.shape[ax]) == int(v.shape[ax]):
        scale = scale[tuple(sl)]
    return Q8Weight(values=values, scale=scale)


def shard_input_channels(w: Weight, rank: int, world: int, axis: int) -> Q8Weight:
    """Row-parallel shard: contraction axis ``axis`` split, scales replicated."""
    q = _q8(w, "weight")
    v = q.values
    ax = axis % v.dim()
    sl = [slice(None)] * v.dim()
    sl[ax] = _span(int(v.shape[ax]), rank, world, "input channels")
    return Q8Weight(values=v[tuple(sl)], scale=q.scale)


def shard_dense_swiglu(gate_w: Weight, up_w: Weight, down_w: Weight, rank: int, world: int):
    """Qwen3 dense MLP shards: gate/up ``[D, I]`` split on I, down ``[I, D]`` split on I."""
    return (
        shard_output_channels(gate_w, rank, world, -1),
        shard_output_channels(up_w, rank, world, -1),
        shard_input_channels(down_w, rank, world, -2),
    )


def shard_gemma_mlp(gating_w: Weight, linear_w: Weight, rank: int, world: int, *, transpose_gating_einsum: bool):
    """Gemma3 MLP shards: gating ``[2, H, D]`` (or ``[2, D, H]``) split on H, linear ``[H, D]`` on H."""
    g = shard_output_channels(gating_w, rank, world, 1 if transpose_gating_einsum else 2)
    return g, shard_input_channels(linear_w, rank, world, 0)


def shard_experts(ffn_gate: Weight, ffn_up: Weight, ffn_down: Weight, rank: int, world: int):
    """Expert-parallel shards: experts ``[r*E/R, (r+1)*E/R)`` of ``[E, ...]`` weights and scales
    (``Q8Weight`` or pre-packed ``Q8Tiled``, whose groups are the experts)."""
    from kappa_b200.qwen3.quant import Q8Tiled

    out = []
    for w in (ffn_gate, ffn_up, ffn_down):
        if isinstance(w, Q8Tiled):
            sl = _span(int(w.kshape[0]), rank, world, "experts")
            scale = w.scale[sl] if w.scale.dim() == len(w.kshape) else w.scale
            out.append(Q8Tiled(tiled=w.tiled[sl], scale=scale, kshape=(sl.stop - sl.start,) + tuple(w.kshape[1:]),
                               in_axis=w.in_axis))
            continue
        q = _q8(w, "expert weight")
        sl = _span(int(q.values.shape[0]), rank, world, "experts")
        scale = q.scale[sl] if q.scale.dim() == q.values.dim() else q.scale
        out.append(Q8Weight(values=q.values[sl], scale=scale))
    return tuple(out)


def _allreduce_to_bf16(partial: torch.Tensor, group) -> torch.Tensor:
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial.to(torch.bfloat16)


def _dense_tp_call(x: torch.Tensor, gate, up, down, hidden: int, act: int, ctx: "TPContext", keep) -> torch.Tensor:
    """One ``kw8_dense_ffn_tp`` call: this rank's shards, partials summed over NVLink."""
    from kappa_b200 import _dense

    b, t, d = x.shape
    T = b * t
    if d != ctx.d or T > ctx.max_tokens:
        raise ValueError(f"TPContext holds {ctx.max_tokens} rows of {ctx.d}, got {T} rows of {d}")
    _dense.check_x(x, d)
    xc = x.contiguous()
    lib = _lib.load()
    out = torch.empty((b, t, d), dtype=torch.bfloat16, device=x.device)
    ws = torch.empty(int(lib.kw8_dense_ffn_tp_workspace_size(T, d, hidden)), dtype=torch.uint8, device=x.device)
    # epoch 0: the device-side call count (calls may be captured in a CUDA graph)
    _lib.check(lib.kw8_dense_ffn_tp(xc.data_ptr(), T, d, hidden, gate, up, down, act, out.data_ptr(),
                                    ctypes.byref(ctx.peers), 0, ws.data_ptr(), ws.numel(), _lib.stream_of(x)))
    del keep
    return out


def swiglu_ffn_tp(x: torch.Tensor, gate_shard: Weight, up_shard: Weight, down_shard: Weight, *, group=None,
                  ctx: "TPContext | None" = None):
    """Tensor-parallel kappa/qwen3/ffn.py:swiglu_ffn over this rank's shards.

    With ``ctx`` (a :class:`TPContext`) the layer is one library call that
    sums the ranks' fp32 partials over NVLink; without, an NCCL all-reduce.
    """
    from kappa_b200.qwen3.ffn import swiglu_ffn

    if ctx is not None:
        g, u, dn = (kmajor(w, -2, n) for w, n in ((gate_shard, "gate_w"), (up_shard, "up_w"), (down_shard, "down_w")))
        return _dense_tp_call(x, g.struct(), u.struct(), dn.struct(), int(g.shape[-2]), _lib.ACT_SILU, ctx,
                              (g, u, dn))
    partial = swiglu_ffn(x, gate_shard, up_shard, down_shard, out_dtype=torch.float32)
    return _allreduce_to_bf16(partial, group)


def feed_forward_tp(x: torch.Tensor, gating_shard: Weight, linear_shard: Weight, *, transpose_gating_einsum: bool,
                    group=None, ctx: "TPContext | None" = None):
    """Tensor-parallel kappa/gemma3/ffn.py:feed_forward over this rank's shards (``ctx``: see swiglu_ffn_tp)."""
    from kappa_b200.gemma3.ffn import feed_forward

    if ctx is not None:
        g = kmajor(gating_shard, -1 if transpose_gating_einsum else -2, "gating_w")
        lw = kmajor(linear_shard, -2, "linear_w")
        hidden = int(g.shape[1])
        return _dense_tp_call(x, g.struct(0), g.struct(hidden), lw.struct(), hidden, _lib.ACT_GELU_TANH, ctx, (g, lw))
    partial = feed_forward(x, gating_shard, linear_shard, transpose_gating_einsum=transpose_gating_einsum,
                           out_dtype=torch.float32)
    return _allreduce_to_bf16(partial, group)


class MoEOps(Protocol):
    """The per-rank compute steps of the MoE layer (see module docstring)."""

    def route(self, x_flat: torch.Tensor, router_w: Weight, num_experts: int, k: int): ...

    def permute(self, idx: torch.Tensor, num_experts: int, capacity: int | None): ...

    def gather(self, x_flat: torch.Tensor, sorted_token: torch.Tensor, rows: int) -> torch.Tensor: ...

    def experts(self, xs: torch.Tensor, group_offsets: torch.Tensor, gate: Weight, up: Weight,
                down: Weight) -> torch.Tensor: ...

    def combine(self, ys: torch.Tensor, inv_pos: torch.Tensor, w: torch.Tensor, d: int) -> torch.Tensor: ...


class KernelMoEOps:
    """MoEOps on the B200 kernels (the staged C-ABI entry points)."""

    def route(self, x_flat, router_w, num_experts, k):
        from kappa_b200.qwen3 import ffn_moe

        _, idx, w = ffn_moe.route_logits(x_flat.unsqueeze(0), router_w, num_experts=num_experts,
                                         num_experts_per_tok=k)
        return idx, w

    def permute(self, idx, num_experts, capacity):
        from kappa_b200.qwen3 import ffn_moe

        return ffn_moe.permute(idx, num_experts, capacity)

    def gather(self, x_flat, sorted_token, rows):
        return x_flat.index_select(0, sorted_token[:rows].long())

    def experts(self, xs, group_offsets, gate, up, down):
        from kappa_b200.qwen3 import ffn_moe

        if xs.shape[0] == 0:
            return torch.empty_like(xs)
        return ffn_moe.expert_ffn(xs, group_offsets, gate, up, down)

    def combine(self, ys, inv_pos, w, d):
        from kappa_b200.qwen3 import ffn_moe

        return ffn_moe.combine(ys, inv_pos, w, d)


def regroup_index(counts: torch.Tensor) -> torch.Tensor:
    """Index that reorders rows received source-major into local-expert-major order.

    ``counts[s][j]``: rows from source rank s for local expert j.  Received
    rows are laid out ``for s: for j``; the result ``perm`` satisfies
    ``regrouped = received[perm]`` with regrouped laid out ``for j: for s``.
    """
    c = counts.to(torch.int64)
    world, e_loc = c.shape
    flat_src = c.reshape(-1)
    src_start = (torch.cumsum(flat_src, 0) - flat_src).reshape(world, e_loc)
    lengths = c.t().reshape(-1)
    dst_start = torch.cumsum(lengths, 0) - lengths
    total = int(lengths.sum())
    shift = src_start.t().reshape(-1) - dst_start
    return torch.arange(total, device=c.device) + torch.repeat_interleave(shift, lengths, output_size=total)


def _moe_args(cfg, x: torch.Tensor):
    if not cfg.use_moe:
        raise ValueError("moe_swiglu_ffn requires cfg.use_moe")
    if x.dim() != 3:
        raise ValueError(f"x must be [B, T, D], got shape {tuple(x.shape)}")
    b, t, d = (int(s) for s in x.shape)
    capacity = None
    if cfg.moe_impl == "fixed_capacity":
        from kappa_b200.qwen3.ffn_moe import fixed_capacity

        if cfg.moe_capacity_factor <= 0:
            raise ValueError("fixed_capacity requires cfg.moe_capacity_factor > 0")
        capacity = fixed_capacity(cfg, b * t)
    return b, t, d, capacity


def _as_i64(v):
    return [int(a) - (1 << 64) if int(a) >= (1 << 63) else int(a) for a in v]


class _SharedBuffers:
    """Device buffers every rank of a group allocates (zero-filled, CUDA IPC)
    and maps from every other rank.  ``peer_ptrs[b]`` is a device int64
    tensor of the ``world`` addresses of buffer ``b`` as this rank sees them;
    ``own[b]`` is this rank's own address.  Collective construction and
    :meth:`close`."""

    def __init__(self, sizes, group, device):
        self.group = group
        self.world, self.rank = _world(group)
        lib = _lib.load()
        hsize = int(lib.kw8_ipc_handle_size())
        self.own = []
        handles = []
        for nbytes in sizes:
            ptr = ctypes.c_void_p()
            h = ctypes.create_string_buffer(hsize)
            _lib.check(lib.kw8_ipc_alloc(max(int(nbytes), 16), ctypes.byref(ptr), h))
            self.own.append(ptr.value)
            handles.append(h.raw)
        allh = [None] * self.world
        dist.all_gather_object(allh, handles, group=group)
        self._opened = []
        peers = [[] for _ in sizes]
        for r, hs in enumerate(allh):
            for b in range(len(sizes)):
                if r == self.rank:
                    peers[b].append(self.own[b])
                else:
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.kw8_ipc_open(ctypes.create_string_buffer(hs[b], hsize), ctypes.byref(ptr)))
                    self._opened.append(ptr.value)
                    peers[b].append(ptr.value)
        self.peer_ptrs = [torch.tensor(_as_i64(v), dtype=torch.int64, device=device) for v in peers]
        self.closed = False

    def close(self, device):
        if self.closed:
            return
        lib = _lib.load()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)
        for p in self._opened:
            lib.kw8_ipc_close(ctypes.c_void_p(p))
        dist.barrier(group=self.group)
        for p in self.own:
            lib.kw8_ipc_free(ctypes.c_void_p(p))
        self.closed = True


class EPContext:
    """Buffers of the NVLink expert-parallel path for one process group.

    Each rank allocates a receive buffer for every row the other ranks could
    send it (``world * max_tokens * k`` rows of ``d``) and a return buffer
    for its own routed rows, shares both with CUDA IPC and maps the other
    ranks' buffers; the decode step (``moe_swiglu_ffn_ep_decode``) sums its
    partials through an exchange buffer of ``decode_tokens`` rows.
    Collective: every rank constructs it with the same arguments and calls
    :meth:`close` (also collective) when done.
    """

    def __init__(self, *, max_tokens: int, d: int, k: int, hidden: int, num_experts: int, group=None,
                 dedup: bool = True, return_format: str = "f16", decode_tokens: int = 256):
        self.group = group
        self.world, self.rank = _world(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.max_tokens, self.d, self.k, self.hidden, self.num_experts = max_tokens, d, k, hidden, num_experts
        self.decode_tokens = decode_tokens
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        self.recv_rows = self.world * max_tokens * k
        self.out_rows = max_tokens * k
        # Shared buffers (zero-filled): receive rows, return rows, counts
        # [2][world][E + world] int32, phase flags [3][world] uint32, and for
        # the deduplicated step: token rows [world * max_tokens][d], pair
        # records (int32 row + fp32 weight per received pair), partial sums
        # [world][max_tokens][d] in `return_format`: "f16" (fp16 rows scaled
        # by a per-row power of two, + a fp32 scale per row: bf16's traffic,
        # relative error per partial up to 2^-11), "f32" (the source rounds
        # each output once, as one GPU does) or "bf16" (up to 2^-9);
        # and the decode exchange buffer [2][world][decode_tokens][d] fp32.
        fmts = {"bf16": _lib.RET_BF16, "f32": _lib.RET_F32, "f16": _lib.RET_F16_SCALED}
        if return_format not in fmts:
            raise ValueError(f"return_format must be one of {sorted(fmts)}, got {return_format!r}")
        self.return_format = return_format
        pairs = self.world * max_tokens * k
        ret_row = d * (4 if return_format == "f32" else 2) + (4 if return_format == "f16" else 0)
        sizes = (self.recv_rows * d * 2, self.out_rows * d * 2, 2 * self.world * (num_experts + self.world) * 4,
                 (3 * self.world + 3) * 4, self.world * max_tokens * d * 2, pairs * 8,
                 self.world * max_tokens * ret_row, 2 * self.world * decode_tokens * d * 4)
        self._bufs = _SharedBuffers(sizes, group, self.device)
        (self.peer_recv, self.peer_out, self.peer_counts, self.peer_flags, self.peer_rows, self.peer_meta,
         self.peer_ret, self.peer_red) = self._bufs.peer_ptrs
        (self.recv_ptr, self.out_ptr, self.counts_ptr, self.flags_ptr, self.rows_ptr, self.meta_ptr,
         self.ret_ptr, self.red_ptr) = self._bufs.own
        self.dedup = dedup
        self.peers = _lib.KW8EpPeers(
            self.world, self.rank, max_tokens, self.peer_recv.data_ptr(), self.peer_out.data_ptr(),
            self.peer_counts.data_ptr(), self.peer_flags.data_ptr(), self.recv_ptr, self.out_ptr,
            self.counts_ptr, self.flags_ptr,
            self.peer_rows.data_ptr() if dedup else None, self.peer_meta.data_ptr() if dedup else None,
            self.peer_ret.data_ptr() if dedup else None, self.rows_ptr if dedup else None,
            self.meta_ptr if dedup else None, self.ret_ptr if dedup else None, fmts[return_format],
            self.peer_red.data_ptr(), self.red_ptr, decode_tokens)
        self.epoch = 0  # calls of the fused steps so far (the group's phase tag)
        self.ep_ws = torch.empty(
            int(lib.kw8_moe_ffn_ep_workspace_size(max_tokens, d, hidden, num_experts, k, self.world)),
            dtype=torch.uint8, device=self.device)
        self.dec_ws = torch.empty(
            int(lib.kw8_moe_ffn_ep_decode_workspace_size(decode_tokens, d, hidden, num_experts, k)),
            dtype=torch.uint8, device=self.device)
        # Staged path (kw8_ep_dispatch / kw8_ep_return + collectives).
        self.ys_loc = torch.empty((self.recv_rows, d), dtype=torch.bfloat16, device=self.device)
        e_loc = num_experts // self.world
        self.ws = torch.empty(int(lib.kw8_moe_expert_ffn_workspace_size(self.recv_rows, d, hidden, e_loc)),
                              dtype=torch.uint8, device=self.device)
        self.loc_off = torch.empty(e_loc + 1, dtype=torch.int32, device=self.device)
        self.counts = torch.empty((self.world, num_experts), dtype=torch.int32, device=self.device)
        self.flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        # Every rank's buffers (flags included) are zero before anyone signals.
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    @property
    def closed(self) -> bool:
        return self._bufs.closed

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch & 0xFFFFFFFF

    def sync(self):
        """Orders the phases across ranks on the current stream (a one-element all-reduce)."""
        dist.all_reduce(self.flag, group=self.group)

    def close(self):
        """Collective: unmaps the other ranks' buffers, then frees this rank's."""
        self._bufs.close(self.device)


class TPContext:
    """The exchange buffer and phase flags of one-call tensor-parallel FFNs
    (``kw8_dense_ffn_tp``) for a process group: every rank's fp32 partial of
    up to ``max_tokens`` rows of ``d`` goes to every rank over NVLink.
    Collective construction and :meth:`close`."""

    def __init__(self, *, max_tokens: int, d: int, group=None):
        self.group = group
        self.world, self.rank = _world(group)
        self.max_tokens, self.d = max_tokens, d
        self.device = torch.device("cuda", torch.cuda.current_device())
        # flags [3][world] + the device call counter and two CTA counters of the
        # exchange kernel; exchange slots [2][world][max_tokens][d] fp32
        self._bufs = _SharedBuffers(((3 * self.world + 3) * 4, 2 * self.world * max_tokens * d * 4), group,
                                    self.device)
        self.peer_flags, self.peer_red = self._bufs.peer_ptrs
        self.flags_ptr, self.red_ptr = self._bufs.own
        self.peers = _lib.KW8EpPeers(
            self.world, self.rank, max_tokens, None, None, None, self.peer_flags.data_ptr(), None, None, None,
            self.flags_ptr, None, None, None, None, None, None, 0, self.peer_red.data_ptr(), self.red_ptr,
            max_tokens)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def close(self):
        self._bufs.close(self.device)


def _moe_ep_p2p(x, router_w, gate_local, up_local, down_local, *, cfg, ctx: EPContext, capacity,
                staged: bool = False):
    from kappa_b200.qwen3 import ffn_moe

    lib = _lib.load()
    b, t, d = (int(s) for s in x.shape)
    T = b * t
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    if T > ctx.max_tokens or d != ctx.d or k != ctx.k or e != ctx.num_experts:
        raise ValueError("EPContext was made for other shapes")
    e_loc = e // ctx.world
    g, u, dn = (kmajor(w, -2, n) for w, n in ((gate_local, "ffn_gate"), (up_local, "ffn_up"),
                                               (down_local, "ffn_down")))
    i = int(g.shape[-2])
    if int(g.shape[0]) != e_loc or i != ctx.hidden:
        raise ValueError("local expert weights do not match the EPContext")
    xc = x.contiguous()
    stream = _lib.stream_of(x)
    if not staged:
        # One call: device-side counts exchange and phase flags, no host
        # round trip and no collective library.
        r = kmajor(router_w, -2, "router_w")
        out = torch.empty((b, t, d), dtype=torch.bfloat16, device=x.device)
        _lib.check(lib.kw8_moe_ffn_ep(
            xc.data_ptr(), T, d, i, e, k, -1 if capacity is None else int(capacity), r.struct(), g.struct(),
            u.struct(), dn.struct(), out.data_ptr(), ctypes.byref(ctx.peers), ctx.next_epoch(),
            ctx.ep_ws.data_ptr(), ctx.ep_ws.numel(), stream))
        del r, g, u, dn
        return out
    _, idx, w = ffn_moe.route_logits(xc, router_w, num_experts=e, num_experts_per_tok=k)
    st, inv, sizes, offs = ffn_moe.permute(idx, e, capacity)
    dist.all_gather_into_tensor(ctx.counts, sizes, group=ctx.group)
    _lib.check(lib.kw8_ep_dispatch(xc.data_ptr(), T * k, d, st.data_ptr(), offs.data_ptr(), ctx.counts.data_ptr(),
                                   ctx.world, ctx.rank, e, ctx.peer_recv.data_ptr(), stream))
    ctx.sync()
    _lib.check(lib.kw8_ep_local_offsets(ctx.counts.data_ptr(), ctx.world, ctx.rank, e, ctx.loc_off.data_ptr(),
                                        stream))
    _lib.check(lib.kw8_moe_expert_ffn(ctx.recv_ptr, ctx.recv_rows, d, i, e_loc, ctx.loc_off.data_ptr(), g.struct(),
                                      u.struct(), dn.struct(), ctx.ys_loc.data_ptr(), ctx.ws.data_ptr(),
                                      ctx.ws.numel(), stream))
    _lib.check(lib.kw8_ep_return(ctx.ys_loc.data_ptr(), ctx.recv_rows, d, ctx.counts.data_ptr(), ctx.world,
                                 ctx.rank, e, ctx.peer_out.data_ptr(), stream))
    ctx.sync()
    out = torch.empty((b, t, d), dtype=torch.bfloat16, device=x.device)
    _lib.check(lib.kw8_moe_combine(ctx.out_ptr, inv.data_ptr(), w.contiguous().data_ptr(), T, k, d,
                                   out.data_ptr(), stream))
    del g, u, dn
    return out


def moe_swiglu_ffn_ep(x: torch.Tensor, router_w: Weight, gate_local: Weight, up_local: Weight, down_local: Weight,
                      *, cfg, group=None, ops: MoEOps | None = None, ctx: EPContext | None = None,
                      staged: bool = False) -> torch.Tensor:
    """Expert-parallel MoE layer over this rank's tokens ``x`` ``[B, T, D]`` (prefill).

    ``gate_local`` / ``up_local`` / ``down_local`` hold this rank's E/R experts
    (``shard_experts``); ``router_w`` is the full router.  Returns the same
    ``[B, T, D]`` bf16 as the single-GPU layer on ``x`` with every expert.
    With ``ctx`` (an :class:`EPContext` of this group) the rows move over
    NVLink with the B200 kernels: by default the whole layer is one library
    call (``kw8_moe_ffn_ep``: counts exchange and phase order by flags in the
    peers' memory); ``staged=True`` runs the same movement as separate calls
    ordered by NCCL collectives.  Without ``ctx``: NCCL all-to-allv.
    """
    if ctx is not None and ops is None:
        _, _, _, capacity = _moe_args(cfg, x)
        return _moe_ep_p2p(x, router_w, gate_local, up_local, down_local, cfg=cfg, ctx=ctx, capacity=capacity,
                           staged=staged)
    ops = ops or KernelMoEOps()
    world, rank = _world(group)
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    if e % world:
        raise ValueError(f"{e} experts do not split over {world} ranks")
    e_loc = e // world
    b, t, d, capacity = _moe_args(cfg, x)
    x_flat = x.reshape(b * t, d)
    idx, w = ops.route(x_flat, router_w, e, k)
    sorted_token, inv_pos, sizes, offsets = ops.permute(idx, e, capacity)
    kept = int(offsets[e])
    xs = ops.gather(x_flat, sorted_token, kept)
    # Per-expert counts: rank r receives the counts of its experts from every source.
    send_counts = sizes.to(torch.int64).contiguous()
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    per_src = recv_counts.reshape(world, e_loc)
    send_split = send_counts.reshape(world, e_loc).sum(1).tolist()
    recv_split = per_src.sum(1).tolist()
    recv_rows = xs.new_empty((sum(recv_split), d))
    dist.all_to_all_single(recv_rows, xs, output_split_sizes=recv_split, input_split_sizes=send_split, group=group)
    perm = regroup_index(per_src)
    xs_loc = recv_rows.index_select(0, perm)
    per_exp = per_src.sum(0)
    loc_off = torch.zeros(e_loc + 1, dtype=torch.int32, device=x.device)
    loc_off[1:] = torch.cumsum(per_exp, 0).to(torch.int32)
    ys_loc = ops.experts(xs_loc, loc_off, gate_local, up_local, down_local)
    recv_y = torch.empty_like(ys_loc)
    recv_y.index_copy_(0, perm, ys_loc)
    ys = xs.new_empty((kept, d))
    dist.all_to_all_single(ys, recv_y, output_split_sizes=send_split, input_split_sizes=recv_split, group=group)
    return ops.combine(ys, inv_pos, w, d).reshape(b, t, d)


def moe_swiglu_ffn_ep_decode(x: torch.Tensor, router_w: Weight, gate_local: Weight, up_local: Weight,
                             down_local: Weight, *, cfg, group=None, ops: MoEOps | None = None,
                             ctx: EPContext | None = None) -> torch.Tensor:
    """Expert-parallel MoE layer for small, replicated batches (decode).

    Every rank passes the same ``x``; each adds its local experts' weighted
    outputs into an fp32 partial and the partials are summed over the group.
    With ``ctx`` (an :class:`EPContext`) the whole step is one library call
    (``kw8_moe_ffn_ep_decode``: the partials cross NVLink with peer stores
    and a flag phase, no host synchronisation); otherwise the staged steps
    of ``ops`` and an NCCL all-reduce (this form also runs on CPU ranks).
    """
    if ctx is not None and ops is None:
        b, t, d, capacity = _moe_args(cfg, x)
        e, k = cfg.num_experts, cfg.num_experts_per_tok
        T = b * t
        if T > ctx.decode_tokens or d != ctx.d or e != ctx.num_experts:
            raise ValueError("EPContext was made for other shapes")
        e_loc = e // ctx.world
        g, u, dn = (kmajor(w, -2, n) for w, n in ((gate_local, "ffn_gate"), (up_local, "ffn_up"),
                                                   (down_local, "ffn_down")))
        if int(g.shape[0]) != e_loc:
            raise ValueError("local expert weights do not match the EPContext")
        r = kmajor(router_w, -2, "router_w")
        lib = _lib.load()
        xc = x.contiguous()
        out = torch.empty((b, t, d), dtype=torch.bfloat16, device=x.device)
        _lib.check(lib.kw8_moe_ffn_ep_decode(
            xc.data_ptr(), T, d, int(g.shape[-2]), e, k, -1 if capacity is None else int(capacity), r.struct(),
            g.struct(), u.struct(), dn.struct(), out.data_ptr(), ctypes.byref(ctx.peers), ctx.next_epoch(),
            ctx.dec_ws.data_ptr(), ctx.dec_ws.numel(), _lib.stream_of(x)))
        del r, g, u, dn
        return out
    ops = ops or KernelMoEOps()
    world, rank = _world(group)
    e, k = cfg.num_experts, cfg.num_experts_per_tok
    if e % world:
        raise ValueError(f"{e} experts do not split over {world} ranks")
    e_loc = e // world
    b, t, d, capacity = _moe_args(cfg, x)
    x_flat = x.reshape(b * t, d)
    idx, w = ops.route(x_flat, router_w, e, k)
    sorted_token, inv_pos, sizes, offsets = ops.permute(idx, e, capacity)
    kept = int(offsets[e])
    xs = ops.gather(x_flat, sorted_token, kept)
    bounds = offsets[rank * e_loc: (rank + 1) * e_loc + 1].to(torch.int64)
    lo, hi = (int(v) for v in bounds[[0, -1]].tolist())
    ys = torch.zeros((kept, d), dtype=torch.bfloat16, device=x.device)
    if hi > lo:
        loc_off = (bounds - lo).to(torch.int32)
        ys[lo:hi] = ops.experts(xs[lo:hi].contiguous(), loc_off, gate_local, up_local, down_local)
    partial = ops.combine(ys, inv_pos, w, d).to(torch.float32)
    return _allreduce_to_bf16(partial, group).reshape(b, t, d)
