"""ctypes binding of ``libkappa_w8.so`` (the C ABI in ``include/kappa_w8.h``).

The shared library is built in-tree (``kappa_b200/build.py``) and loaded
from this package's directory.  There is no fallback: if the library is
missing, or no CUDA device is present, calls raise.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libkappa_w8.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# kw8_status
KW8_OK = 0
KW8_ERR_INVALID_ARG = -1
KW8_ERR_UNSUPPORTED = -2
KW8_ERR_CUDA = -3
KW8_ERR_WORKSPACE = -4
KW8_ERR_DEVICE_TIMEOUT = -5

# kw8_dtype
DT_F32 = 0
DT_BF16 = 1

# kw8_act
ACT_GELU_TANH = 0
ACT_SILU = 1

# kw8_layout
LAYOUT_KMAJOR = 0
LAYOUT_TILED = 1

# kw8_ret_format (partial sums of the expert-parallel return)
RET_BF16 = 0
RET_F32 = 1
RET_F16_SCALED = 2

# kw8_norm_kind
NORM_GEMMA = 0  # x * rsqrt(mean(x^2) + eps) * (1 + scale)
NORM_QWEN = 1  # x * rsqrt(mean(x^2) + eps) * scale

# kw8_set_option
OPT_GEMM_PATH = 0  # 0 auto, 1 tensor core, 2 weight streaming (decode kernel)
OPT_TOKEN_TILE = 1  # 0 auto, 16..256
OPT_DETERMINISTIC = 2  # 1: the MoE combine sums each token's k rows in a fixed order
OPT_TC_PAIR = 3  # tensor-core GEMM over SM pairs: 0 auto (one-CTA), 1 never, 2 whenever the tile allows
OPT_EP_TIMING = 4  # 1: CUDA events at the phase boundaries of kw8_moe_ffn_ep (kw8_ep_phase_times)


class KW8Error(RuntimeError):
    """A libkappa_w8 call failed; ``code`` is the kw8_status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"kappa_w8 error {code}: {message}")
        self.code = code


class KW8Weight(ctypes.Structure):
    """``kw8_weight`` (include/kappa_w8.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("scale_dtype", ctypes.c_int32),
        ("per_channel", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class KW8BlockNorms(ctypes.Structure):
    """``kw8_block_norms`` (include/kappa_w8.h): the norms around a block's FFN."""

    _fields_ = [
        ("pre_scale", ctypes.c_void_p),
        ("post_scale", ctypes.c_void_p),
        ("scale_dtype", ctypes.c_int32),
        ("kind", ctypes.c_int32),
        ("eps", ctypes.c_float),
    ]


class KW8EpPeers(ctypes.Structure):
    """``kw8_ep_peers`` (include/kappa_w8.h): an expert-parallel group seen from one rank."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("max_tokens", ctypes.c_int64),
        ("recv", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("counts", ctypes.c_void_p),
        ("flags", ctypes.c_void_p),
        ("own_recv", ctypes.c_void_p),
        ("own_out", ctypes.c_void_p),
        ("own_counts", ctypes.c_void_p),
        ("own_flags", ctypes.c_void_p),
        ("rows", ctypes.c_void_p),
        ("meta", ctypes.c_void_p),
        ("ret", ctypes.c_void_p),
        ("own_rows", ctypes.c_void_p),
        ("own_meta", ctypes.c_void_p),
        ("own_ret", ctypes.c_void_p),
        ("ret_format", ctypes.c_int32),
        ("red", ctypes.c_void_p),
        ("own_red", ctypes.c_void_p),
        ("red_rows", ctypes.c_int64),
    ]


_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t

# name -> (restype, argtypes); exactly the functions include/kappa_w8.h declares.
SIGNATURES: dict[str, tuple] = {
    "kw8_last_error": (ctypes.c_char_p, []),
    "kw8_abi_version": (_i32, []),
    "kw8_device_status": (ctypes.c_int, [ctypes.POINTER(_i32), _vp]),
    "kw8_set_option": (ctypes.c_int, [_i32, _i64]),
    "kw8_quantize_workspace_size": (_sz, [_i64, _i64]),
    "kw8_quantize": (
        ctypes.c_int,
        [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _sz, _vp],
    ),
    "kw8_dequantize": (ctypes.c_int, [KW8Weight, _i64, _i64, _i64, _i32, _vp, _vp]),
    "kw8_packed_weight_bytes": (_sz, [_i64, _i64, _i64]),
    "kw8_pack_weight": (ctypes.c_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "kw8_unpack_weight": (ctypes.c_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "kw8_dense_ffn_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kw8_dense_ffn": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, KW8Weight, KW8Weight, KW8Weight, _i32, _i32, _vp, _vp, _sz, _vp],
    ),
    "kw8_linear_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kw8_linear": (ctypes.c_int, [_vp, _vp, _i64, _i64, _i64, KW8Weight, _i32, _vp, _vp, _sz, _vp]),
    "kw8_embed_gather": (ctypes.c_int, [_vp, _i64, KW8Weight, _i64, _i64, _i32, _vp, _vp]),
    "kw8_rms_norm": (ctypes.c_int, [_vp, _i64, _i64, _vp, _i32, _i32, ctypes.c_float, _vp, _vp]),
    "kw8_dense_block_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kw8_dense_block": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, KW8Weight, KW8Weight, KW8Weight, _i32, ctypes.POINTER(KW8BlockNorms), _vp, _vp,
         _sz, _vp],
    ),
    "kw8_moe_block_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "kw8_moe_block": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i32, _i64, KW8Weight, KW8Weight, KW8Weight, KW8Weight,
         ctypes.POINTER(KW8BlockNorms), _vp, _vp, _sz, _vp],
    ),
    "kw8_moe_route": (ctypes.c_int, [_vp, _i64, _i64, _i64, _i32, KW8Weight, _vp, _vp, _vp, _vp]),
    "kw8_moe_topk": (ctypes.c_int, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    "kw8_moe_permute": (ctypes.c_int, [_vp, _i64, _i32, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "kw8_moe_permute_workspace_size": (ctypes.c_size_t, [_i64]),
    "kw8_ipc_handle_size": (ctypes.c_size_t, []),
    "kw8_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _vp]),
    "kw8_ipc_free": (ctypes.c_int, [_vp]),
    "kw8_ipc_open": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "kw8_ipc_close": (ctypes.c_int, [_vp]),
    "kw8_ep_dispatch": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _i64, _vp, _vp]),
    "kw8_ep_return": (ctypes.c_int, [_vp, _i64, _i64, _vp, _i32, _i32, _i64, _vp, _vp]),
    "kw8_ep_local_offsets": (ctypes.c_int, [_vp, _i32, _i32, _i64, _vp, _vp]),
    "kw8_moe_ffn_ep_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32, _i32]),
    "kw8_moe_ffn_ep": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i32, _i64, KW8Weight, KW8Weight, KW8Weight, KW8Weight, _vp,
         ctypes.POINTER(KW8EpPeers), ctypes.c_uint32, _vp, _sz, _vp],
    ),
    "kw8_moe_ffn_ep_decode_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "kw8_moe_ffn_ep_decode": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i32, _i64, KW8Weight, KW8Weight, KW8Weight, KW8Weight, _vp,
         ctypes.POINTER(KW8EpPeers), ctypes.c_uint32, _vp, _sz, _vp],
    ),
    "kw8_dense_ffn_tp_workspace_size": (_sz, [_i64, _i64, _i64]),
    "kw8_dense_ffn_tp": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, KW8Weight, KW8Weight, KW8Weight, _i32, _vp, ctypes.POINTER(KW8EpPeers),
         ctypes.c_uint32, _vp, _sz, _vp],
    ),
    "kw8_ep_phase_times": (ctypes.c_int, [_vp, _i32]),
    "kw8_ep_barrier": (ctypes.c_int, [ctypes.POINTER(KW8EpPeers), _i32, ctypes.c_uint32, _i32, _vp]),
    "kw8_moe_permute_ws": (ctypes.c_int, [_vp, _i64, _i32, _i64, _i64, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "kw8_moe_expert_ffn_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "kw8_moe_expert_ffn": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _vp, KW8Weight, KW8Weight, KW8Weight, _vp, _vp, _sz, _vp],
    ),
    "kw8_moe_combine": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i32, _i64, _vp, _vp]),
    "kw8_moe_ffn_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "kw8_moe_ffn": (
        ctypes.c_int,
        [
            _vp, _i64, _i64, _i64, _i64, _i32, _i64,
            KW8Weight, KW8Weight, KW8Weight, KW8Weight, _vp, _vp, _sz, _vp,
        ],
    ),
    "kw8_moe_ffn_noalloc": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i32, _i64, KW8Weight, KW8Weight, KW8Weight, KW8Weight, _vp, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m kappa_b200.build`"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().kw8_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    """Raise for a non-zero kw8_status (ValueError for bad arguments)."""
    if rc == KW8_OK:
        return
    msg = last_error()
    if rc in (KW8_ERR_INVALID_ARG, KW8_ERR_UNSUPPORTED):
        raise ValueError(f"kappa_w8: {msg}")
    raise KW8Error(rc, msg)


def stream_of(t: torch.Tensor) -> int:
    """Handle of torch's current stream on ``t``'s device."""
    return torch.cuda.current_stream(t.device).cuda_stream


def device_status(t: torch.Tensor) -> int:
    """Read and clear the device status word (synchronises the stream)."""
    v = _i32(0)
    check(load().kw8_device_status(ctypes.byref(v), stream_of(t)))
    return int(v.value)


def set_option(option: int, value: int) -> None:
    check(load().kw8_set_option(option, value))


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (kappa_b200 has no CPU path)")
