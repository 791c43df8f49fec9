"""kw8_moe_ffn_noalloc: the MoE layer for callers that cannot allocate.

Some callers cannot hand the library a workspace — for example a custom-call
handler that is given only its input and output buffers, or a program whose
device memory belongs to an allocator it cannot reach where it calls this
library.  ``kw8_moe_ffn_noalloc`` serves them from a fixed 16 MiB scratch
array inside the library.  These tests call it through the C ABI and check
it against the workspace entry point, ``kw8_moe_ffn``, within the parity
tolerance the other GPU tests use, on two calls in a row (the second call
finds the first call's leftovers in the shared scratch).

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import pytest
import torch

from helpers import TOL, parity, to_np
from kappa_b200 import _lib
from kappa_b200.qwen3.quant import kmajor, quantize_weight

pytestmark = pytest.mark.gpu

D, I, E, K = 2048, 768, 128, 8  # Qwen3-30B-A3B MoE layer shape


def _layer(seed: int):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def q8(shape):
        w = torch.randn(shape, generator=g, device=dev) * 0.02
        return kmajor(quantize_weight(w, per_channel=True, scale_dtype=torch.float32), -2)

    return [q8((D, E)), q8((E, D, I)), q8((E, D, I)), q8((E, I, D))], g


def _x(g, T):
    return torch.randn((T, D), generator=g, device="cuda").to(torch.bfloat16)


def _with_workspace(lib, x, ws_structs, stream):
    T = x.shape[0]
    out = torch.empty_like(x)
    n = int(lib.kw8_moe_ffn_workspace_size(T, D, I, E, K))
    ws = torch.empty(n, dtype=torch.uint8, device=x.device)
    _lib.check(lib.kw8_moe_ffn(x.data_ptr(), T, D, I, E, K, -1, *ws_structs, out.data_ptr(),
                               ws.data_ptr(), n, stream))
    return out


def _no_alloc(lib, x, ws_structs, stream):
    out = torch.empty_like(x)
    _lib.check(lib.kw8_moe_ffn_noalloc(x.data_ptr(), x.shape[0], D, I, E, K, -1, *ws_structs,
                                       out.data_ptr(), stream))
    return out


def test_no_alloc_matches_workspace_entry_point():
    lib = _lib.load()
    weights, g = _layer(seed=7)
    structs = [w.struct() for w in weights]
    stream = torch.cuda.current_stream().cuda_stream
    for T in (64, 256):
        x = _x(g, T)
        ref = to_np(_with_workspace(lib, x, structs, stream)).astype("float32")
        first = to_np(_no_alloc(lib, x, structs, stream)).astype("float32")
        second = to_np(_no_alloc(lib, x, structs, stream)).astype("float32")
        parity(first, ref, tol=TOL)
        parity(second, ref, tol=TOL)
    assert _lib.device_status(x) == 0


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    weights, g = _layer(seed=8)
    structs = [w.struct() for w in weights]
    x = _x(g, 4096)  # needs ~200 MB of scratch, far above the 16 MiB built in
    out = torch.empty_like(x)
    rc = lib.kw8_moe_ffn_noalloc(x.data_ptr(), 4096, D, I, E, K, -1, *structs, out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.KW8_ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
