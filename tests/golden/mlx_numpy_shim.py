"""A numpy stand-in for the handful of MLX calls the reference's gated-delta
files make, so that those files can be imported and run unchanged on a host
without MLX (test infrastructure only: used by ``make_golden.py``).

Only the operations that the reference's hot-path modules call are provided:

* ``mlx_lean_moe/model/qwen3_5/gated_delta.py``: ``mx.exp``, ``nn.softplus``,
  ``mx.repeat``, ``mx.stack``, ``mx.default_device``/``mx.gpu``/
  ``mx.metal.is_available`` (always "no Metal", so the ops path runs);
* ``mlx_lean_moe/model/qwen3_5/linear_attention.py``: ``mx.concatenate``,
  ``mx.conv1d`` (depthwise, cross-correlation, no padding), ``mx.split``,
  ``mx.fast.rms_norm``, ``mx.sigmoid``, ``nn.silu``;
* ``mlx_lean_moe/cache/recurrent_cache.py``: ``mx.zeros``;
* ``mlx_lean_moe/model/rope.py``: ``mx.fast.rope`` (non-traditional: feature
  i pairs with i + dims / 2; position = offset + index along the sequence);
* ``mlx_lean_moe/model/qwen3_5/attention.py``:
  ``mx.fast.scaled_dot_product_attention`` (grouped-query heads, the causal
  mask aligned to the last query: query i of L sees keys j <= T - L + i),
  ``mx.sigmoid``;
* ``mlx_lean_moe/cache/kv_cache.py``: ``mx.zeros``, ``mx.concatenate``.

Each follows MLX's documented semantics for float32 inputs; no other dtype is
exercised by the golden generator.
"""

from __future__ import annotations

import importlib.util
import sys
import types

import numpy as np


def _rms_norm(x, weight, eps):
    x = np.asarray(x)
    ms = np.mean(np.square(x.astype(np.float32)), axis=-1, keepdims=True)
    out = x.astype(np.float32) / np.sqrt(ms + np.float32(eps))
    if weight is not None:
        out = out * np.asarray(weight, dtype=np.float32)
    return out.astype(x.dtype)


def _conv1d(x, w, stride=1, padding=0, dilation=1, groups=1):
    """MLX layout: x (N, L, C_in), w (C_out, K, C_in // groups); output
    (N, L - K + 1, C_out); out[n, t, c] = sum_j x[n, t + j, c] * w[c, j, 0]
    for the depthwise case (groups == C_in == C_out)."""

    x = np.asarray(x)
    w = np.asarray(w)
    assert stride == 1 and padding == 0 and dilation == 1
    n, length, c_in = x.shape
    c_out, kernel, per_group = w.shape
    assert groups == c_in == c_out and per_group == 1, "depthwise only"
    out_len = length - kernel + 1
    out = np.zeros((n, out_len, c_out), dtype=np.result_type(x, w))
    for j in range(kernel):
        out += x[:, j : j + out_len, :] * w[None, None, :, j, 0]
    return out


def _split(a, indices, axis=0):
    return np.split(np.asarray(a), indices, axis=axis)


def _sigmoid(x):
    x = np.asarray(x)
    return (1.0 / (1.0 + np.exp(-x))).astype(x.dtype)


def _silu(x):
    x = np.asarray(x)
    return (x * _sigmoid(x)).astype(x.dtype)


def _softplus(x):
    x = np.asarray(x)
    return np.logaddexp(np.zeros((), dtype=x.dtype), x).astype(x.dtype)


def _rope(x, dims, traditional=False, base=10000.0, scale=1.0, offset=0):
    """(B, H, L, D): rotate features [0, dims) pairwise (i, i + dims / 2) by
    angle (offset + l) * scale * base ** (-2 i / dims); the rest pass."""

    assert not traditional
    x = np.asarray(x)
    out = x.astype(np.float64).copy()
    half = dims // 2
    inv = base ** (-np.arange(half, dtype=np.float64) * 2.0 / dims)
    pos = (offset + np.arange(x.shape[-2], dtype=np.float64)) * scale
    ang = pos[:, None] * inv[None, :]
    cos, sin = np.cos(ang), np.sin(ang)
    a, b = out[..., :half].copy(), out[..., half:dims].copy()
    out[..., :half] = a * cos - b * sin
    out[..., half:dims] = b * cos + a * sin
    return out.astype(x.dtype)


def _sdpa(q, k, v, scale, mask=None):
    """q (B, H, L, D), k/v (B, Hkv, T, D): softmax(scale q k^T [+ causal]) v,
    query head h reading key/value head h // (H / Hkv)."""

    q, k, v = (np.asarray(a) for a in (q, k, v))
    bsz, h, length, _ = q.shape
    hkv, t = k.shape[1], k.shape[2]
    rep = h // hkv
    kk = np.repeat(k.astype(np.float64), rep, axis=1)
    vv = np.repeat(v.astype(np.float64), rep, axis=1)
    s = np.einsum("bhld,bhtd->bhlt", q.astype(np.float64), kk) * scale
    if mask is not None:
        assert mask == "causal"
        allowed = np.arange(t)[None, :] <= (t - length + np.arange(length))[:, None]
        s = np.where(allowed[None, None], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhlt,bhtd->bhld", p, vv).astype(q.dtype)


def build_modules() -> dict[str, types.ModuleType]:
    core = types.ModuleType("mlx.core")
    core.array = np.ndarray
    core.Dtype = np.dtype
    core.float32 = np.float32
    core.float16 = np.float16
    core.float64 = np.float64
    core.exp = np.exp
    core.repeat = np.repeat
    core.stack = np.stack
    core.concatenate = np.concatenate
    core.split = _split
    core.sigmoid = _sigmoid
    core.conv1d = _conv1d
    core.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype)
    core.eval = lambda *a, **k: None
    core.cpu = "cpu"
    core.gpu = "gpu"
    core.default_device = lambda: "cpu"
    core.metal = types.SimpleNamespace(is_available=lambda: False)
    core.fast = types.SimpleNamespace(rms_norm=_rms_norm, rope=_rope, scaled_dot_product_attention=_sdpa)

    nn = types.ModuleType("mlx.nn")
    nn.silu = _silu
    nn.softplus = _softplus

    mlx = types.ModuleType("mlx")
    mlx.core = core
    mlx.nn = nn
    return {"mlx": mlx, "mlx.core": core, "mlx.nn": nn}


def load_reference_modules(src_root: str) -> dict[str, types.ModuleType]:
    """Import the reference's hot-path modules from ``src_root`` (the
    reference's ``src`` directory) on top of the numpy shim. Package
    ``__init__`` files are skipped: they would import the whole model stack."""

    sys.modules.update(build_modules())
    pkg_dirs = {
        "mlx_lean_moe": "mlx_lean_moe",
        "mlx_lean_moe.cache": "mlx_lean_moe/cache",
        "mlx_lean_moe.model": "mlx_lean_moe/model",
        "mlx_lean_moe.model.qwen3_5": "mlx_lean_moe/model/qwen3_5",
    }
    for name, rel in pkg_dirs.items():
        pkg = types.ModuleType(name)
        pkg.__path__ = [f"{src_root}/{rel}"]
        sys.modules[name] = pkg

    def load(name: str, rel: str) -> types.ModuleType:
        spec = importlib.util.spec_from_file_location(name, f"{src_root}/{rel}")
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
        return module

    modules = {}
    modules["config"] = load("mlx_lean_moe.config", "mlx_lean_moe/config.py")
    modules["qconfig"] = load(
        "mlx_lean_moe.model.qwen3_5.config", "mlx_lean_moe/model/qwen3_5/config.py"
    )
    modules["moe_block"] = load(
        "mlx_lean_moe.model.moe_block", "mlx_lean_moe/model/moe_block.py"
    )
    modules["recurrent_cache"] = load(
        "mlx_lean_moe.cache.recurrent_cache", "mlx_lean_moe/cache/recurrent_cache.py"
    )
    modules["metal"] = load(
        "mlx_lean_moe.model.qwen3_5._gated_delta_metal",
        "mlx_lean_moe/model/qwen3_5/_gated_delta_metal.py",
    )
    modules["gated_delta"] = load(
        "mlx_lean_moe.model.qwen3_5.gated_delta",
        "mlx_lean_moe/model/qwen3_5/gated_delta.py",
    )
    modules["linear_attention"] = load(
        "mlx_lean_moe.model.qwen3_5.linear_attention",
        "mlx_lean_moe/model/qwen3_5/linear_attention.py",
    )
    modules["kv_cache"] = load("mlx_lean_moe.cache.kv_cache", "mlx_lean_moe/cache/kv_cache.py")
    modules["rope"] = load("mlx_lean_moe.model.rope", "mlx_lean_moe/model/rope.py")
    modules["attention"] = load(
        "mlx_lean_moe.model.qwen3_5.attention", "mlx_lean_moe/model/qwen3_5/attention.py"
    )
    return modules
