"""ctypes binding of ``libgdn_oracle.so`` (the C restatement in
``gdn_oracle.c``) -- TEST INFRASTRUCTURE ONLY, used as the checker at sizes
where the numpy oracle would be too slow."""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgdn_oracle.so")
_lib = None


def build() -> str:
    """Compile ``libgdn_oracle.so`` with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        f = lib.gdn_oracle_scan_varlen
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        f.argtypes = [p, p, p, p, p, p, i64, i64, i64, i64, i64, ctypes.c_int, p, p, p, ctypes.c_int]
        f.restype = ctypes.c_int
        _lib = lib
    return _lib


def scan_varlen(q, k, v, g, beta, cu_seqlens, states, g_is_log=False, n_threads=None):
    """Float64 recurrence over packed sequences (see ``gdn_oracle.c``).
    Inputs are converted to contiguous float32; returns float32
    ``(y (N, Hv, Dv), states (B, Hv, Dv, Dk))``."""

    lib = _load()
    q, k, v, g, beta, states = (
        np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta, states)
    )
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int64)
    n, hk, dk = q.shape
    hv, dv = v.shape[1], v.shape[2]
    n_seq = len(cu) - 1
    assert states.shape == (n_seq, hv, dv, dk)
    assert int(cu[-1]) == n and k.shape == q.shape and g.shape == (n, hv) == beta.shape
    y = np.zeros((n, hv, dv), np.float32)
    out = np.zeros_like(states)
    if n_threads is None:
        n_threads = os.cpu_count() or 1
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = lib.gdn_oracle_scan_varlen(
        ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(cu), n_seq, hk, hv, dk, dv,
        int(bool(g_is_log)), ptr(states), ptr(y), ptr(out), int(n_threads),
    )
    if rc != 0:
        raise RuntimeError(f"gdn_oracle_scan_varlen failed with status {rc}")
    return y, out
