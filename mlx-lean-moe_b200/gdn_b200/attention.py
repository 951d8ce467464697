"""The softmax-attention layer on B200 (the reference's ``Qwen3_5Attention``,
``qw/attention.py:17-99``) and its growing key/value cache
(``cache/kv_cache.py:28-102``).

``Qwen3_5Attention`` keeps the reference's constructor and call: the
projections go through ``quantized_linear`` (dense or affine-quantized
weights), everything between them -- the q/k RMS norms, the rotary
embedding of the leading ``rotary_dim`` features, the cache append, the
grouped-query causal attention and the output gate -- is one
``gdn_attention`` call into libgdn_b200.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .gated_delta import _DTYPES, _require_cuda, _stream
from .quantized import LinearWeights, QuantScheme, as_linear, concat_rows, quantized_linear


class GrowingKVCache:
    """``cache/kv_cache.py:28-102`` on the GPU: head-major ``(kv_heads,
    tokens, head_dim)`` buffers growing in 256-token blocks up to
    ``max_context``, the hard limit (appending past it raises rather than
    wraps)."""

    def __init__(self, max_context: int, num_kv_heads: int, head_dim: int, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None) -> None:
        if max_context <= 0:
            raise ValueError(f"max_context must be positive, got {max_context}")
        self.capacity = max_context
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._keys = torch.zeros((num_kv_heads, 0, head_dim), dtype=dtype, device=self.device)
        self._values = torch.zeros((num_kv_heads, 0, head_dim), dtype=dtype, device=self.device)
        self._written = 0

    @property
    def allocated_size(self) -> int:
        return self._keys.shape[1]

    @property
    def size(self) -> int:
        return self._written

    def reserve(self, n_new: int) -> int:
        """Make room for ``n_new`` more tokens (the reference's growth rule,
        ``kv_cache.py:65-78``); returns the cache length after them."""

        end = self._written + n_new
        if end > self.capacity:
            raise IndexError(f"GrowingKVCache exceeded its capacity of {self.capacity} tokens")
        if end > self.allocated_size:
            allocated = min(self.capacity, ((end + 255) // 256) * 256)
            grow = (self._keys.shape[0], allocated, self._keys.shape[2])
            keys = torch.zeros(grow, dtype=self._keys.dtype, device=self.device)
            values = torch.zeros(grow, dtype=self._values.dtype, device=self.device)
            keys[:, : self._written] = self._keys[:, : self._written]
            values[:, : self._written] = self._values[:, : self._written]
            self._keys, self._values = keys, values
        return end

    def commit(self, end: int) -> None:
        self._written = end

    def append_many(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Append a head-major ``(heads, tokens, dim)`` batch (checked before
        either buffer is touched)."""

        if keys.ndim != 3 or values.shape != keys.shape:
            raise ValueError("keys and values must have matching (heads, tokens, dim) shapes")
        if keys.shape[0] != self._keys.shape[0] or keys.shape[2] != self._keys.shape[2]:
            raise ValueError("keys and values do not match the cache head count or dimension")
        end = self.reserve(keys.shape[1])
        self._keys[:, self._written:end] = keys
        self._values[:, self._written:end] = values
        self._written = end

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        self.append_many(key[:, None, :], value[:, None, :])

    def state(self) -> tuple[torch.Tensor, torch.Tensor]:
        n = self._written
        return self._keys[:, :n, :], self._values[:, :n, :]


@dataclass(frozen=True)
class AttentionShape:
    """``qw/config.py``: head counts, head size, rotary width, RoPE base."""

    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rotary_dim: int
    rope_theta: float


def attention_core(qg: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm: torch.Tensor,
                   k_norm: torch.Tensor, shape: AttentionShape, eps: float, cache: GrowingKVCache) -> torch.Tensor:
    """``qw/attention.py:56-96`` between the projections, for ``L`` new tokens:
    ``qg (L, heads * 2 * head_dim)`` (per head: queries | gate), ``k``/``v``
    ``(L, kv_heads * head_dim)``; advances ``cache`` by ``L``. Returns the
    gated attention output ``(L, heads * head_dim)`` in ``qg``'s dtype."""

    device = _require_cuda(qg, k, v, q_norm, k_norm)
    n = qg.shape[0]
    h, hkv, hd = shape.num_attention_heads, shape.num_key_value_heads, shape.head_dim
    if qg.ndim != 2 or qg.shape[1] != h * 2 * hd or k.shape != (n, hkv * hd) or v.shape != k.shape:
        raise ValueError("qg must be (L, heads * 2 * head_dim) and k, v (L, kv_heads * head_dim)")
    if qg.dtype not in (torch.float32, torch.bfloat16) or k.dtype != qg.dtype or v.dtype != qg.dtype:
        raise ValueError("qg, k and v must share a float32 or bfloat16 dtype")
    if cache._keys.dtype != qg.dtype:
        raise ValueError("the cache dtype must match the activations")
    qg, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (qg, k, v))
    end = cache.reserve(n)
    out = torch.empty(n, h * hd, dtype=qg.dtype, device=device)
    qn, kn = q_norm.float().contiguous(), k_norm.float().contiguous()
    a = _lib.AttnArgs()
    a.n_tokens, a.cache_len, a.capacity = n, end, cache.allocated_size
    a.heads, a.kv_heads, a.head_dim, a.rotary_dim = h, hkv, hd, shape.rotary_dim
    a.rope_base, a.eps, a.scale = float(shape.rope_theta), float(eps), float(hd ** -0.5)
    a.qg, a.qg_stride_t = qg.data_ptr(), qg.stride(0)
    a.k_new, a.k_stride_t = k.data_ptr(), k.stride(0)
    a.v_new, a.v_stride_t = v.data_ptr(), v.stride(0)
    a.q_norm, a.k_norm = qn.data_ptr(), kn.data_ptr()
    a.k_cache, a.v_cache = cache._keys.data_ptr(), cache._values.data_ptr()
    a.act_dtype = _DTYPES[qg.dtype]
    a.out, a.out_stride_t = out.data_ptr(), out.stride(0)
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.gdn_attention_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)), "attention")
        ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes.value
        _lib.check(lib.gdn_attention(ctypes.byref(a), _stream(device)), "attention")
    cache.commit(end)
    return out


class Qwen3_5Attention:
    """``qw/attention.py:17-99``: ``__call__(x, cache)`` takes ``(hidden,)``
    for one decode step or ``(L, hidden)`` and returns the same rank,
    appending to ``cache`` (a ``GrowingKVCache``). Projections are dense
    ``(out, in)`` tensors, ``LinearWeights``, or ``{weight, scales, biases}``
    dicts stored with ``quant`` (the reference's ``config.other_quant``)."""

    def __init__(self, shape: AttentionShape, rms_norm_eps: float, q_proj, q_norm: torch.Tensor, k_proj,
                 k_norm: torch.Tensor, v_proj, o_proj, quant: QuantScheme | None = None) -> None:
        self.shape = shape
        self.eps = rms_norm_eps
        self.q_proj, self.k_proj = as_linear(q_proj, quant), as_linear(k_proj, quant)
        self.v_proj, self.o_proj = as_linear(v_proj, quant), as_linear(o_proj, quant)
        self.q_norm, self.k_norm = q_norm, k_norm
        # One product gives q|gate, k and v when the three share a storage
        # scheme (one GEMV per decode step instead of three).
        parts = (self.q_proj, self.k_proj, self.v_proj)
        self.qkv_proj: LinearWeights | None = concat_rows(list(parts)) if len({p.quant for p in parts}) == 1 else None

    def __call__(self, x: torch.Tensor, cache: GrowingKVCache) -> torch.Tensor:
        if x.ndim not in (1, 2):
            raise ValueError(f"Qwen3_5Attention expects 1-D or 2-D x, got shape {tuple(x.shape)}")
        squeeze = x.ndim == 1
        rows = x[None, :] if squeeze else x
        if self.qkv_proj is not None:
            qkv = quantized_linear(rows, self.qkv_proj)
            s = self.shape
            nq, nkv = s.num_attention_heads * 2 * s.head_dim, s.num_key_value_heads * s.head_dim
            qg, k, v = qkv[:, :nq], qkv[:, nq:nq + nkv], qkv[:, nq + nkv:]
        else:
            qg = quantized_linear(rows, self.q_proj)
            k = quantized_linear(rows, self.k_proj)
            v = quantized_linear(rows, self.v_proj)
        out = attention_core(qg, k, v, self.q_norm, self.k_norm, self.shape, self.eps, cache)
        out = quantized_linear(out, self.o_proj)
        return out[0] if squeeze else out
