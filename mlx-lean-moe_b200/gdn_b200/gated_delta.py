"""The gated-delta operator on B200: the reference's op API over libgdn_b200.

Mirrors ``src/mlx_lean_moe/model/qwen3_5/gated_delta.py`` of the reference
(``qw/`` below): ``forget_gate`` (``qw/gated_delta.py:14-21``),
``gated_delta_step`` (``:24-41``) and ``gated_delta_scan`` (``:44-90``) keep
their names, argument meaning, shape checks and error messages; arrays are
CUDA ``torch`` tensors instead of MLX arrays. Every call runs a CUDA kernel
of libgdn_b200.so; there is no CPU path.

Batched forms the reference does not have (it is single-sequence,
``qw/gated_delta.py:5``) are added for serving and prefill:
``gated_delta_scan_varlen`` (packed sequences with ``cu_seqlens``) and
``gated_delta_decode`` (one token for many sequences, optional state slots).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16, torch.float16: _lib.GDN_F16}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("gdn_b200 operates on CUDA tensors only (no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same CUDA device")
    if device is None:
        raise ValueError("no CUDA tensor given")
    _lib.load()
    return device


def _inner_contiguous(t: torch.Tensor) -> torch.Tensor:
    """Feature dimension contiguous (the reference's kernel copies strided
    inputs, ``qw/_gated_delta_metal.py:43``); other strides pass through."""
    return t if t.stride(-1) == 1 else t.contiguous()


def _qkv_common(q, k, v):
    if q.dtype == k.dtype == v.dtype and q.dtype in _DTYPES:
        return q, k, v
    return q.float(), k.float(), v.float()


def _gate(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype in (torch.float32, torch.bfloat16) else t.float()


def forget_gate(a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor, *, log: bool = False) -> torch.Tensor:
    """``qw/gated_delta.py:14-21``: per-value-head decay in (0, 1],
    ``exp(-exp(A_log) * softplus(a + dt_bias))``, float32. ``log=True``
    returns its logarithm (the form the chunked prefill consumes).
    ``a``: ``(..., Hv)``."""

    device = _require_cuda(a, A_log, dt_bias)
    hv = a.shape[-1]
    if A_log.shape != (hv,) or dt_bias.shape != (hv,):
        raise ValueError("A_log and dt_bias must have shape (value_heads,)")
    a2 = a.reshape(-1, hv)
    if a2.stride(-1) != 1 or a.dtype not in _DTYPES:
        a2 = a2.contiguous() if a.dtype in _DTYPES else a2.float().contiguous()
    A = A_log.float().contiguous()
    dt = dt_bias.float().contiguous()
    g = torch.empty(a2.shape, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        st = _lib.load().gdn_forget_gate(
            a2.data_ptr(), _DTYPES[a2.dtype], a2.stride(0), a2.shape[0], hv, A.data_ptr(), dt.data_ptr(),
            g.data_ptr(), _lib.GDN_GATE_LOG if log else _lib.GDN_GATE_MULT, _stream(device),
        )
    _lib.check(st, "forget_gate")
    return g.reshape(a.shape)


def _validate(q, k, v, g, beta, state):
    """The checks of ``qw/gated_delta.py:57-79``, same messages."""

    if q.ndim != 3 or k.shape != q.shape or v.ndim != 3:
        raise ValueError("q/k must have matching (L, key_heads, key_dim) shapes; v must be 3-D")
    length, key_heads, key_dim = q.shape
    _, value_heads, value_dim = v.shape
    if min(length, key_heads, key_dim, value_heads, value_dim) <= 0:
        raise ValueError("gated_delta_scan requires nonempty sequence and head dimensions")
    if v.shape[0] != length or value_heads % key_heads:
        raise ValueError("v must match q's sequence length and have a multiple of its head count")
    if tuple(g.shape) != (length, value_heads) or beta.shape != g.shape:
        raise ValueError("g and beta must have shape (L, value_heads)")
    if tuple(state.shape) != (value_heads, value_dim, key_dim):
        raise ValueError("state must have shape (value_heads, value_dim, key_dim)")


def _scan_args(q, k, v, g, beta, state_in, state_out, out, n_seqs, cu_seqlens, g_is_log, algo):
    a = _lib.ScanArgs()
    a.n_tokens = q.shape[0]
    a.n_seqs = n_seqs
    a.cu_seqlens = cu_seqlens.data_ptr() if cu_seqlens is not None else None
    a.hk, a.dk = q.shape[1], q.shape[2]
    a.hv, a.dv = v.shape[1], v.shape[2]
    a.q, a.q_stride_t, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_t, a.k_stride_h = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_t, a.v_stride_h = v.data_ptr(), v.stride(0), v.stride(1)
    a.g, a.g_stride_t = g.data_ptr(), g.stride(0)
    a.beta, a.beta_stride_t = beta.data_ptr(), beta.stride(0)
    a.state_in = state_in.data_ptr() if state_in is not None else None
    a.state_out = state_out.data_ptr()
    a.out = out.data_ptr()
    a.qkv_dtype = _DTYPES[q.dtype]
    a.gate_dtype = _DTYPES[g.dtype]
    a.out_dtype = _DTYPES[out.dtype]
    a.gate_kind = _lib.GDN_GATE_LOG if g_is_log else _lib.GDN_GATE_MULT
    a.algo = _lib.ALGOS[algo]
    return a


def _prepare_gates(g, beta):
    g, beta = _gate(g), _gate(beta)
    if g.dtype != beta.dtype:
        g, beta = g.float(), beta.float()
    if g.stride(-1) != 1:
        g = g.contiguous()
    if beta.stride(-1) != 1:
        beta = beta.contiguous()
    return g, beta


def _run_scan(args, device, what):
    lib = _lib.load()
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(lib.gdn_scan_workspace_size(ctypes.byref(args), ctypes.byref(ws_bytes)), what)
    workspace = None
    if ws_bytes.value:
        workspace = torch.empty(ws_bytes.value, dtype=torch.uint8, device=device)
        args.workspace = workspace.data_ptr()
        args.workspace_bytes = ws_bytes.value
    _lib.check(lib.gdn_scan(ctypes.byref(args), _stream(device)), what)
    return workspace


def gated_delta_scan(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor,
    *,
    use_kernel: bool = True,
    g_is_log: bool = False,
    algo: str = "auto",
) -> tuple[torch.Tensor, torch.Tensor]:
    """``qw/gated_delta.py:44-90``: the recurrence over ``L`` positions of one
    sequence. q/k ``(L, Hk, Dk)``, v ``(L, Hv, Dv)``, g/beta ``(L, Hv)``,
    state ``(Hv, Dv, Dk)``. ``g`` is the multiplicative decay (the
    reference's convention) unless ``g_is_log``. Returns ``(y (L, Hv, Dv),
    new_state (Hv, Dv, Dk))``; the input state is not modified.

    The state is carried in float32 whatever its dtype (the reference's
    cache keeps it float32, ``cache/recurrent_cache.py:28-32``); outputs take
    the dtype the reference's promotion gives (float32 when any input is
    float32). ``use_kernel`` is accepted for signature compatibility: there
    is only the CUDA path."""

    del use_kernel
    _validate(q, k, v, g, beta, state)
    device = _require_cuda(q, k, v, g, beta, state)
    result_dtype = torch.result_type(torch.empty((), dtype=q.dtype), torch.empty((), dtype=state.dtype))
    for t in (k, v, g, beta):
        result_dtype = torch.promote_types(result_dtype, t.dtype)
    q, k, v = _qkv_common(_inner_contiguous(q), _inner_contiguous(k), _inner_contiguous(v))
    g, beta = _prepare_gates(g, beta)
    state_in = state.float().contiguous()
    state_out = torch.empty_like(state_in)
    y = torch.empty(v.shape, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        args = _scan_args(q, k, v, g, beta, state_in, state_out, y, 1, None, g_is_log, algo)
        _run_scan(args, device, "gated_delta_scan")
    if result_dtype != torch.float32:
        return y.to(result_dtype), state_out.to(result_dtype)
    return y, state_out


def gated_delta_step(q, k, v, g, beta, state):
    """``qw/gated_delta.py:24-41``: one step, q/k ``(Hv, Dk)`` already
    repeated out to the value heads, v ``(Hv, Dv)``, g/beta ``(Hv,)``, state
    ``(Hv, Dv, Dk)``. Returns ``(y (Hv, Dv), new_state)``."""

    if q.ndim != 2 or k.shape != q.shape or v.ndim != 2 or v.shape[0] != q.shape[0]:
        raise ValueError("q/k must be (Hv, Dk) and v (Hv, Dv)")
    y, new_state = gated_delta_decode(
        q[None], k[None], v[None], g[None], beta[None], state[None].float().contiguous(), inplace=False
    )
    return y[0], new_state[0]


def gated_delta_scan_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor | None,
    cu_seqlens: torch.Tensor | None = None,
    *,
    g_is_log: bool = False,
    algo: str = "auto",
    out_dtype: torch.dtype = torch.float32,
    state_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed multi-sequence scan. q/k ``(N, Hk, Dk)``, v ``(N, Hv, Dv)``,
    g/beta ``(N, Hv)``; ``cu_seqlens`` int64 ``(B + 1,)`` on the device (or
    None for one sequence); state float32 ``(B, Hv, Dv, Dk)`` or None for
    zeros. ``state_out`` may be ``state`` itself (in-place cache update).
    Returns ``(y (N, Hv, Dv), state_out)``."""

    device = _require_cuda(q, k, v, g, beta, state, cu_seqlens)
    if q.ndim != 3 or k.shape != q.shape or v.ndim != 3 or v.shape[0] != q.shape[0]:
        raise ValueError("q/k must be (N, Hk, Dk) and v (N, Hv, Dv)")
    n_seqs = 1 if cu_seqlens is None else cu_seqlens.numel() - 1
    hv, dv, dk = v.shape[1], v.shape[2], q.shape[2]
    if tuple(g.shape) != (q.shape[0], hv) or beta.shape != g.shape:
        raise ValueError("g and beta must have shape (N, value_heads)")
    if cu_seqlens is not None and (cu_seqlens.dtype != torch.int64 or cu_seqlens.ndim != 1 or n_seqs < 1):
        raise ValueError("cu_seqlens must be a 1-D int64 tensor of B + 1 offsets")
    if state is not None and (tuple(state.shape) != (n_seqs, hv, dv, dk) or state.dtype != torch.float32
                              or not state.is_contiguous()):
        raise ValueError("state must be a contiguous float32 (B, Hv, Dv, Dk) tensor")
    q, k, v = _qkv_common(_inner_contiguous(q), _inner_contiguous(k), _inner_contiguous(v))
    g, beta = _prepare_gates(g, beta)
    if state_out is None:
        state_out = torch.empty((n_seqs, hv, dv, dk), dtype=torch.float32, device=device)
    if out is None:
        out = torch.empty(v.shape, dtype=out_dtype, device=device)
    with torch.cuda.device(device):
        args = _scan_args(q, k, v, g, beta, state, state_out, out, n_seqs, cu_seqlens, g_is_log, algo)
        _run_scan(args, device, "gated_delta_scan_varlen")
    return out, state_out


def gated_delta_decode(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor,
    *,
    g_is_log: bool = False,
    state_slots: torch.Tensor | None = None,
    inplace: bool = True,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One token for each of B sequences. q/k ``(B, Hk, Dk)``, v ``(B, Hv,
    Dv)``, g/beta ``(B, Hv)``; state float32 ``(B, Hv, Dv, Dk)``, or a pool
    ``(S, Hv, Dv, Dk)`` indexed by int32 ``state_slots (B,)`` (distinct
    slots). With ``inplace`` (the cache update of ``qw/linear_attention.py:120``)
    the state is advanced in place, else a new state is returned.
    Returns ``(y (B, Hv, Dv), state)``."""

    device = _require_cuda(q, k, v, g, beta, state, state_slots)
    if q.ndim != 3 or k.shape != q.shape or v.ndim != 3 or v.shape[0] != q.shape[0]:
        raise ValueError("q/k must be (B, Hk, Dk) and v (B, Hv, Dv)")
    bsz, hv, dv, dk = q.shape[0], v.shape[1], v.shape[2], q.shape[2]
    if tuple(g.shape) != (bsz, hv) or beta.shape != g.shape:
        raise ValueError("g and beta must have shape (B, value_heads)")
    n_rows = state.shape[0]
    if tuple(state.shape[1:]) != (hv, dv, dk) or state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("state must be a contiguous float32 (B or slots, Hv, Dv, Dk) tensor")
    if state_slots is None and n_rows != bsz:
        raise ValueError("state must have one row per sequence when state_slots is None")
    if state_slots is not None and (state_slots.dtype != torch.int32 or state_slots.shape != (bsz,)):
        raise ValueError("state_slots must be an int32 (B,) tensor")
    q, k, v = _qkv_common(_inner_contiguous(q), _inner_contiguous(k), _inner_contiguous(v))
    g, beta = _prepare_gates(g, beta)
    state_out = state if inplace else torch.empty_like(state)
    if out is None:
        out = torch.empty((bsz, hv, dv), dtype=out_dtype, device=device)
    if not inplace and state_slots is not None:
        state_out.copy_(state)
    with torch.cuda.device(device):
        d = _lib.DecodeArgs()
        d.base = _scan_args(q, k, v, g, beta, state, state_out, out, bsz, None, g_is_log, "auto")
        d.state_slots = state_slots.data_ptr() if state_slots is not None else None
        d.n_slots = n_rows if state_slots is not None else 0
        _lib.check(_lib.load().gdn_decode(ctypes.byref(d), _stream(device)), "gated_delta_decode")
    return out, state_out


class DecodePlan:
    """``gated_delta_decode`` prepared once for fixed buffers.

    A server's decode loop writes each step's q, k, v, g, beta into the same
    tensors and advances the same state; ``DecodePlan`` validates them and
    builds the argument block once, and ``run()`` only launches (on the
    current stream), the state advancing in place as with
    ``gated_delta_decode(..., inplace=True)``.  The buffers must be usable as
    given (q/k/v of one supported dtype and g/beta float32 or bfloat16 alike,
    feature dimensions contiguous): a plan never copies, so later writes to
    the caller's tensors are what ``run()`` reads."""

    def __init__(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        g: torch.Tensor,
        beta: torch.Tensor,
        state: torch.Tensor,
        *,
        g_is_log: bool = False,
        state_slots: torch.Tensor | None = None,
        out_dtype: torch.dtype = torch.float32,
        out: torch.Tensor | None = None,
    ) -> None:
        device = _require_cuda(q, k, v, g, beta, state, state_slots, out)
        if q.ndim != 3 or k.shape != q.shape or v.ndim != 3 or v.shape[0] != q.shape[0]:
            raise ValueError("q/k must be (B, Hk, Dk) and v (B, Hv, Dv)")
        bsz, hv, dv = q.shape[0], v.shape[1], v.shape[2]
        if tuple(g.shape) != (bsz, hv) or beta.shape != g.shape:
            raise ValueError("g and beta must have shape (B, value_heads)")
        n_rows = state.shape[0]
        if tuple(state.shape[1:]) != (hv, dv, q.shape[2]) or state.dtype != torch.float32 or not state.is_contiguous():
            raise ValueError("state must be a contiguous float32 (B or slots, Hv, Dv, Dk) tensor")
        if state_slots is None and n_rows != bsz:
            raise ValueError("state must have one row per sequence when state_slots is None")
        if state_slots is not None and (state_slots.dtype != torch.int32 or state_slots.shape != (bsz,)):
            raise ValueError("state_slots must be an int32 (B,) tensor")
        if _qkv_common(q, k, v)[0] is not q or any(t.stride(-1) != 1 for t in (q, k, v)):
            raise ValueError("DecodePlan needs q, k, v of one supported dtype with contiguous feature dimensions")
        g2, beta2 = _prepare_gates(g, beta)
        if g2 is not g or beta2 is not beta:
            raise ValueError("DecodePlan needs g and beta of one dtype (float32 or bfloat16), last dim contiguous")
        if out is None:
            out = torch.empty((bsz, hv, dv), dtype=out_dtype, device=device)
        elif tuple(out.shape) != (bsz, hv, dv) or not out.is_contiguous():
            raise ValueError("out must be a contiguous (B, Hv, Dv) tensor")
        d = _lib.DecodeArgs()
        d.base = _scan_args(q, k, v, g, beta, state, state, out, bsz, None, g_is_log, "auto")
        d.state_slots = state_slots.data_ptr() if state_slots is not None else None
        d.n_slots = n_rows if state_slots is not None else 0
        self._args = d
        self._argp = ctypes.byref(d)
        self._lib = _lib.load()
        self._keep = (q, k, v, g, beta, state, state_slots)
        self.device = device
        self.out = out
        self.state = state

    def run(self) -> torch.Tensor:
        """One decode step on the current stream; returns ``out``."""
        _lib.check(self._lib.gdn_decode(self._argp, torch.cuda.current_stream(self.device).cuda_stream),
                   "gated_delta_decode")
        return self.out


def check_device_errors(device: torch.device | None = None) -> None:
    """Synchronise the current stream and raise if a bounded device wait of
    the library gave up since the last check."""

    device = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        _lib.check(_lib.load().gdn_check_device_errors(_stream(device)), "device error check")
