"""The C ABI library loads on a CPU-only host and exports what the header declares."""

from __future__ import annotations

import os
import re

import kappa_b200._lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "kappa_w8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(kw8_\w+)\s*\(", src))


def test_header_matches_binding():
    assert _declared() == set(L.SIGNATURES)


def test_library_exports_every_symbol():
    lib = L.load()
    for name in _declared():
        assert hasattr(lib, name), name


def test_cpu_only_queries():
    lib = L.load()
    assert lib.kw8_abi_version() == 3
    n = lib.kw8_moe_ffn_workspace_size(4096, 2048, 768, 128, 8)
    # permuted rows xs (32768 x 2048 bf16), h (32768 x 768 bf16) and the
    # fp32 combine buffer (4096 x 2048) dominate
    assert n > 32768 * 2048 * 2 + 32768 * 768 * 2 + 4096 * 2048 * 4
    assert lib.kw8_dense_ffn_workspace_size(256, 2560, 10240) >= 256 * 10240 * 2
    assert lib.kw8_quantize_workspace_size(128, 768) >= 128 * 768 * 4


def test_workspace_sizes_do_not_depend_on_the_path_option():
    """A workspace sized under one OPT_GEMM_PATH value serves the others."""
    lib = L.load()
    sizes = []
    try:
        for opt in (0, 1, 2):
            L.set_option(L.OPT_GEMM_PATH, opt)
            sizes.append(([lib.kw8_moe_ffn_workspace_size(T, 2048, 768, 128, 8) for T in (1, 16, 64, 256, 4096)],
                          [lib.kw8_dense_ffn_workspace_size(T, 2560, 10240) for T in (1, 16, 64, 256)]))
    finally:
        L.set_option(L.OPT_GEMM_PATH, 0)
    assert sizes[0] == sizes[1] == sizes[2]


def test_invalid_arguments_fail_before_any_launch():
    lib = L.load()
    w = L.KW8Weight(None, None, 0, 0)
    rc = lib.kw8_moe_ffn(None, 4, 16, 16, 4, 2, -1, w, w, w, w, None, None, 0, None)
    assert rc == L.KW8_ERR_INVALID_ARG
    assert "null" in L.last_error()
    assert lib.kw8_set_option(0, 7) == L.KW8_ERR_INVALID_ARG
    assert lib.kw8_set_option(1, 24) == L.KW8_ERR_INVALID_ARG


def test_new_entry_points_reject_bad_arguments_before_any_launch():
    """Null pointers, bad shapes and bad enums of the linear, embedding,
    norm, block, packing and group entry points fail on the host."""
    import ctypes

    lib = L.load()
    w = L.KW8Weight(None, None, 0, 0, 0, 0)
    ok_w = L.KW8Weight(1 << 20, 1 << 20, L.DT_F32, 1, L.LAYOUT_KMAJOR, 0)  # never dereferenced
    assert lib.kw8_linear(None, None, 4, 64, 64, w, L.DT_BF16, None, None, 0, None) == L.KW8_ERR_INVALID_ARG
    assert lib.kw8_linear(1 << 20, None, 4, 64, 64, ok_w, 7, 1 << 20, None, 0, None) == L.KW8_ERR_INVALID_ARG
    bad_layout = L.KW8Weight(1 << 20, 1 << 20, L.DT_F32, 1, 5, 0)
    assert lib.kw8_linear(1 << 20, None, 4, 64, 64, bad_layout, L.DT_BF16, 1 << 20, None, 0, None) == \
        L.KW8_ERR_INVALID_ARG
    assert "layout" in L.last_error()
    assert lib.kw8_embed_gather(None, 4, w, 10, 64, L.DT_BF16, None, None) == L.KW8_ERR_INVALID_ARG
    # D must be a multiple of 8 and at most 16384; the kind must be known
    assert lib.kw8_rms_norm(1 << 20, 4, 12, 1 << 20, L.DT_BF16, L.NORM_GEMMA, 1e-6, 1 << 20, None) == \
        L.KW8_ERR_UNSUPPORTED
    assert lib.kw8_rms_norm(1 << 20, 4, 64, 1 << 20, L.DT_BF16, 9, 1e-6, 1 << 20, None) == L.KW8_ERR_INVALID_ARG
    norms = L.KW8BlockNorms(None, None, L.DT_BF16, L.NORM_QWEN, 1e-6)
    assert lib.kw8_dense_block(1 << 20, 4, 64, 128, ok_w, ok_w, ok_w, L.ACT_SILU, ctypes.byref(norms), 2 << 20,
                               None, 0, None) == L.KW8_ERR_INVALID_ARG
    assert "pre-FFN" in L.last_error()
    assert lib.kw8_moe_block(1 << 20, 4, 64, 32, 8, 2, -1, ok_w, ok_w, ok_w, ok_w, ctypes.byref(norms), 1 << 20,
                             None, 0, None) == L.KW8_ERR_INVALID_ARG  # out aliases h
    assert lib.kw8_pack_weight(1 << 20, 1, 16, 24, 1 << 20, None) == L.KW8_ERR_INVALID_ARG  # K % 16
    assert lib.kw8_packed_weight_bytes(2, 100, 208) == 2 * 7 * 4 * 1024
    peers = L.KW8EpPeers()
    peers.world, peers.rank = 2, 0
    assert lib.kw8_dense_ffn_tp(1 << 20, 4, 64, 128, ok_w, ok_w, ok_w, L.ACT_SILU, 1 << 20, ctypes.byref(peers), 0,
                                None, 0, None) == L.KW8_ERR_INVALID_ARG
    assert "exchange buffer" in L.last_error()
    ms = (ctypes.c_float * 9)()
    assert lib.kw8_ep_phase_times(ms, 0) != L.KW8_OK
