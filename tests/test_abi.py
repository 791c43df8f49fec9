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
