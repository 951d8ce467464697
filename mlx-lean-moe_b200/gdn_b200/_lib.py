"""ctypes binding of libgdn_b200.so (the C ABI declared in include/gdn_api.h,
and the test hooks of include/gdn_testing.h).

The library is the only compute path: if it is missing or CUDA is not usable,
calls raise; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn_b200.so")

GDN_OK, GDN_EINVAL, GDN_EUNSUPPORTED, GDN_ECUDA, GDN_ETIMEOUT = range(5)
GDN_F32, GDN_BF16, GDN_F16 = 0, 1, 2
GDN_GATE_MULT, GDN_GATE_LOG = 0, 1
GDN_ALGO_AUTO, GDN_ALGO_SERIAL, GDN_ALGO_CHUNKED = 0, 1, 2
ALGOS = {"auto": GDN_ALGO_AUTO, "serial": GDN_ALGO_SERIAL, "chunked": GDN_ALGO_CHUNKED}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_enum = ctypes.c_int


class ScanArgs(ctypes.Structure):
    """``gdn_scan_args``."""

    _fields_ = [
        ("n_tokens", _i64), ("n_seqs", _i64), ("cu_seqlens", _p),
        ("hk", _i32), ("hv", _i32), ("dk", _i32), ("dv", _i32),
        ("q", _p), ("q_stride_t", _i64), ("q_stride_h", _i64),
        ("k", _p), ("k_stride_t", _i64), ("k_stride_h", _i64),
        ("v", _p), ("v_stride_t", _i64), ("v_stride_h", _i64),
        ("g", _p), ("g_stride_t", _i64),
        ("beta", _p), ("beta_stride_t", _i64),
        ("state_in", _p), ("state_out", _p), ("out", _p),
        ("qkv_dtype", _enum), ("gate_dtype", _enum), ("out_dtype", _enum),
        ("gate_kind", _enum), ("algo", _enum),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
    ]


class DecodeArgs(ctypes.Structure):
    """``gdn_decode_args``."""

    _fields_ = [("base", ScanArgs), ("state_slots", _p), ("n_slots", _i64)]


class BlockArgs(ctypes.Structure):
    """``gdn_block_args``."""

    _fields_ = [
        ("n_tokens", _i64), ("n_seqs", _i64), ("cu_seqlens", _p),
        ("hk", _i32), ("hv", _i32), ("dk", _i32), ("dv", _i32), ("conv_kernel", _i32),
        ("mixed", _p), ("mixed_stride_t", _i64), ("act_dtype", _enum),
        ("conv_w", _p), ("conv_state_in", _p), ("conv_state_out", _p), ("conv_state_dtype", _enum),
        ("A_log", _p), ("dt_bias", _p), ("norm_w", _p), ("eps", ctypes.c_float),
        ("state_in", _p), ("state_out", _p), ("out", _p), ("algo", _enum),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
    ]


class QLinearArgs(ctypes.Structure):
    """``gdn_qlinear_args``."""

    _fields_ = [
        ("m", _i64), ("n", _i64), ("k", _i64),
        ("x", _p), ("x_stride_m", _i64),
        ("w", _p), ("scales", _p), ("biases", _p),
        ("bits", _i32), ("group_size", _i32),
        ("out", _p), ("out_stride_m", _i64),
    ]


class AttnArgs(ctypes.Structure):
    """``gdn_attn_args``."""

    _fields_ = [
        ("n_tokens", _i64), ("cache_len", _i64), ("capacity", _i64),
        ("heads", _i32), ("kv_heads", _i32), ("head_dim", _i32), ("rotary_dim", _i32),
        ("rope_base", ctypes.c_float), ("eps", ctypes.c_float), ("scale", ctypes.c_float),
        ("qg", _p), ("qg_stride_t", _i64),
        ("k_new", _p), ("k_stride_t", _i64),
        ("v_new", _p), ("v_stride_t", _i64),
        ("q_norm", _p), ("k_norm", _p),
        ("k_cache", _p), ("v_cache", _p),
        ("act_dtype", _enum),
        ("out", _p), ("out_stride_t", _i64),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
    ]


MAX_GATHER_PEERS = 7
IPC_HANDLE_BYTES = 64


class GatherArgs(ctypes.Structure):
    """``gdn_gather_args``."""

    _fields_ = [
        ("hv_total", _i32), ("head0", _i32), ("n_peers", _i32), ("reserved", _i32),
        ("peer_out", _p * MAX_GATHER_PEERS),
    ]


EXPORTS = {
    "gdn_version": (ctypes.c_int, []),
    "gdn_last_error": (ctypes.c_char_p, []),
    "gdn_scan_workspace_size": (_enum, [ctypes.POINTER(ScanArgs), ctypes.POINTER(ctypes.c_size_t)]),
    "gdn_scan": (_enum, [ctypes.POINTER(ScanArgs), _p]),
    "gdn_decode": (_enum, [ctypes.POINTER(DecodeArgs), _p]),
    "gdn_forget_gate": (_enum, [_p, _enum, _i64, _i64, _i32, _p, _p, _p, _enum, _p]),
    "gdn_block_workspace_size": (_enum, [ctypes.POINTER(BlockArgs), ctypes.POINTER(ctypes.c_size_t)]),
    "gdn_fused_block": (_enum, [ctypes.POINTER(BlockArgs), _p]),
    "gdn_fused_block_noalloc": (_enum, [ctypes.POINTER(BlockArgs), _p]),
    "gdn_quantized_linear": (_enum, [ctypes.POINTER(QLinearArgs), _p]),
    "gdn_dequantize": (_enum, [ctypes.POINTER(QLinearArgs), _enum, _p, _p]),
    "gdn_attention_workspace_size": (_enum, [ctypes.POINTER(AttnArgs), ctypes.POINTER(ctypes.c_size_t)]),
    "gdn_attention": (_enum, [ctypes.POINTER(AttnArgs), _p]),
    "gdn_scan_gathered": (_enum, [ctypes.POINTER(ScanArgs), ctypes.POINTER(GatherArgs), _p]),
    "gdn_ipc_export": (_enum, [_p, ctypes.POINTER(ctypes.c_ubyte), ctypes.POINTER(ctypes.c_uint64)]),
    "gdn_ipc_import": (_enum, [ctypes.POINTER(ctypes.c_ubyte), ctypes.c_uint64, ctypes.POINTER(_p)]),
    "gdn_ipc_release": (_enum, [_p, ctypes.c_uint64]),
    "gdn_check_device_errors": (_enum, [_p]),
    "gdn_test_set_wait_limit": (_enum, [ctypes.c_uint64]),
    "gdn_test_inject_fault": (_enum, [_i32]),
}

_lib = None


class GdnError(RuntimeError):
    """A CUDA failure or a device-side timeout reported by the library."""


def load() -> ctypes.CDLL:
    """Load libgdn_b200.so (built in-tree by ``__graft_entry__.build()`` or
    ``make -C mlx-lean-moe_b200/csrc``); raises if it is missing."""

    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libgdn_b200.so not found at {LIB_PATH}: build it with "
                "`make -C mlx-lean-moe_b200/csrc` (no CPU fallback exists)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in EXPORTS.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.gdn_version() != 1:
            raise ImportError("libgdn_b200.so has an unexpected API version")
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Raise for a non-zero gdn_status: ValueError for argument/shape errors
    (as the reference raises before dispatch), GdnError for CUDA/timeouts."""

    if status == GDN_OK:
        return
    msg = load().gdn_last_error().decode(errors="replace")
    if status in (GDN_EINVAL, GDN_EUNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise GdnError(f"{what} failed ({status}): {msg}")
