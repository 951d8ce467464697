"""CPU oracle for the gated-delta path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker: the product path
(``gdn_b200``) never calls it and has no CPU fallback.

Every function restates one piece of the reference (conferencebeefwood46/
mlx-lean-moe) in numpy, citing the file:line it follows. Paths are relative to
the reference project root; ``qw/`` stands for
``src/mlx_lean_moe/model/qwen3_5/``.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own modules
(``qw/gated_delta.py``, ``qw/linear_attention.py``,
``src/mlx_lean_moe/cache/recurrent_cache.py``) unchanged on a numpy stand-in
for MLX, plus the reference's own float64 test recurrence
(``tests/test_gated_delta_metal.py:10-39``), and commits the outputs under
``tests/golden/``. ``tests/test_oracle_golden.py`` checks every function here
against those vectors.
"""

from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------
# Input generators (restated from the reference's tests, same seeds/shapes)
# ---------------------------------------------------------------------------


def metal_test_inputs(length, key_dim=128, value_dim=17, key_heads=2, value_heads=4):
    """``_inputs`` of ``tests/test_gated_delta_metal.py:10-23``: seed 42,
    q L2-normalised and divided by sqrt(Dk), k L2-normalised, v ~ N(0,1),
    g ~ U(0.98, 1) with head 0 forced to 1, beta ~ U(0, 1), state ~ 0.1 N(0,1).
    Returns float32 arrays (q, k, v, g, beta, state)."""

    rng = np.random.default_rng(42)
    q = rng.normal(size=(length, key_heads, key_dim))
    k = rng.normal(size=q.shape)
    q /= np.linalg.norm(q, axis=-1, keepdims=True) * key_dim**0.5
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.normal(size=(length, value_heads, value_dim))
    g = rng.uniform(0.98, 1, size=(length, value_heads))
    g[:, 0] = 1
    beta = rng.uniform(0, 1, size=g.shape)
    state = rng.normal(size=(value_heads, value_dim, key_dim)) * 0.1
    return [a.astype(np.float32) for a in (q, k, v, g, beta, state)]


def gdn_test_inputs(seed, seq_len, hk=2, hv=6, dk=16, dv=8):
    """``_inputs`` of ``tests/test_qwen3_5_gated_delta.py:26-38``: standard
    normals drawn in the order q, k, v, a, b, A_log, dt_bias."""

    rng = np.random.default_rng(seed)

    def f32(*shape):
        return rng.standard_normal(shape).astype(np.float32)

    return {
        "q": f32(seq_len, hk, dk),
        "k": f32(seq_len, hk, dk),
        "v": f32(seq_len, hv, dv),
        "a": f32(seq_len, hv),
        "b": f32(seq_len, hv),
        "A_log": f32(hv),
        "dt_bias": f32(hv),
    }


# ---------------------------------------------------------------------------
# The op (qw/gated_delta.py)
# ---------------------------------------------------------------------------


def softplus(x):
    """``nn.softplus``: log(1 + exp(x)), evaluated without overflow."""
    return np.logaddexp(np.zeros((), dtype=x.dtype), x).astype(x.dtype)


def forget_gate(a, A_log, dt_bias):
    """``qw/gated_delta.py:14-21``: exp(-exp(A_log) * softplus(a + dt_bias)),
    all in float32."""

    a32 = np.asarray(a, np.float32)
    return np.exp(
        -np.exp(np.asarray(A_log, np.float32))
        * softplus(a32 + np.asarray(dt_bias, np.float32))
    ).astype(np.float32)


def forget_gate_log(a, A_log, dt_bias):
    """The log of :func:`forget_gate`, -exp(A_log) * softplus(a + dt_bias),
    float32 (the log-decay form the chunked prefill consumes)."""

    a32 = np.asarray(a, np.float32)
    return (
        -np.exp(np.asarray(A_log, np.float32))
        * softplus(a32 + np.asarray(dt_bias, np.float32))
    ).astype(np.float32)


def gated_delta_step(q, k, v, g, beta, state):
    """``qw/gated_delta.py:24-41``. q/k ``(Hv, Dk)`` already repeated out to
    the value heads; v ``(Hv, Dv)``; g, beta ``(Hv,)``; state
    ``(Hv, Dv, Dk)``. Same operation order as the reference."""

    state = state * g[:, None, None]
    read = (state * k[:, None, :]).sum(axis=-1)
    delta = (v - read) * beta[:, None]
    state = state + k[:, None, :] * delta[:, :, None]
    y = (state * q[:, None, :]).sum(axis=-1)
    return y, state


def validate_scan(q, k, v, g, beta, state):
    """The shape checks of ``qw/gated_delta.py:57-79``, with the reference's
    messages; raises ValueError."""

    if q.ndim != 3 or k.shape != q.shape or v.ndim != 3:
        raise ValueError(
            "q/k must have matching (L, key_heads, key_dim) shapes; v must be 3-D"
        )
    length, key_heads, key_dim = q.shape
    _, value_heads, value_dim = v.shape
    if min(length, key_heads, key_dim, value_heads, value_dim) <= 0:
        raise ValueError(
            "gated_delta_scan requires nonempty sequence and head dimensions"
        )
    if v.shape[0] != length or value_heads % key_heads:
        raise ValueError(
            "v must match q's sequence length and have a multiple of its head count"
        )
    if g.shape != (length, value_heads) or beta.shape != g.shape:
        raise ValueError("g and beta must have shape (L, value_heads)")
    if state.shape != (value_heads, value_dim, key_dim):
        raise ValueError("state must have shape (value_heads, value_dim, key_dim)")


def gated_delta_scan(q, k, v, g, beta, state, dtype=np.float64):
    """``qw/gated_delta.py:44-109`` (validation, then ``_gated_delta_scan_ops``):
    GQA by repeat-interleave of q/k over the value heads (``:97-101``), then
    :func:`gated_delta_step` for each position in order (``:105-107``).

    ``g`` is the multiplicative decay in (0, 1]. Computes in ``dtype``
    (float64 by default, the precision of the reference's own test recurrence
    ``tests/test_gated_delta_metal.py:26-39``). The input state is not
    mutated. Returns ``(y (L, Hv, Dv), state (Hv, Dv, Dk))`` in ``dtype``."""

    validate_scan(q, k, v, g, beta, state)
    q, k, v, g, beta, state = (np.asarray(a).astype(dtype) for a in (q, k, v, g, beta, state))
    repeat = v.shape[-2] // q.shape[-2]
    if repeat > 1:
        q = np.repeat(q, repeat, axis=-2)
        k = np.repeat(k, repeat, axis=-2)
    outputs = []
    for t in range(q.shape[0]):
        y, state = gated_delta_step(q[t], k[t], v[t], g[t], beta[t], state)
        outputs.append(y)
    return np.stack(outputs), state


def reference_f64(inputs):
    """The reference's independent float64 recurrence,
    ``tests/test_gated_delta_metal.py:26-39``, restated (einsum form)."""

    q, k, v, g, beta, state = [np.array(a).astype(np.float64) for a in inputs]
    repeat = v.shape[1] // q.shape[1]
    q, k = np.repeat(q, repeat, axis=1), np.repeat(k, repeat, axis=1)
    output = []
    for t in range(len(q)):
        state *= g[t, :, None, None]
        read = np.einsum("hvk,hk->hv", state, k[t])
        correction = (v[t] - read) * beta[t, :, None]
        state += np.einsum("hv,hk->hvk", correction, k[t])
        output.append(np.einsum("hvk,hk->hv", state, q[t]))
    return np.stack(output), state


def scan_varlen(q, k, v, g, beta, cu_seqlens, states, dtype=np.float64, g_is_log=False):
    """Packed variable-length form: sequence ``i`` owns rows
    ``cu_seqlens[i]:cu_seqlens[i+1]`` of q/k/v/g/beta and ``states[i]``.
    Each sequence is an independent call of :func:`gated_delta_scan` (the
    reference has no batch axis, ``qw/gated_delta.py:5``). A sequence of
    length 0 keeps its state. ``g_is_log`` feeds ``exp(g)`` to the reference
    semantics. Returns ``(y (N, Hv, Dv), states (B, Hv, Dv, Dk))``."""

    n_seq = len(cu_seqlens) - 1
    hv, dv = v.shape[1], v.shape[2]
    y = np.zeros((v.shape[0], hv, dv), dtype=dtype)
    out_states = np.array(states, dtype=dtype, copy=True)
    for i in range(n_seq):
        s, e = int(cu_seqlens[i]), int(cu_seqlens[i + 1])
        if e == s:
            continue
        gi = np.exp(np.asarray(g[s:e], np.float64)) if g_is_log else g[s:e]
        yi, st = gated_delta_scan(q[s:e], k[s:e], v[s:e], gi, beta[s:e], states[i], dtype)
        y[s:e] = yi
        out_states[i] = st
    return y, out_states


# ---------------------------------------------------------------------------
# The layer's prologue / epilogue (qw/linear_attention.py)
# ---------------------------------------------------------------------------


def rms_norm(x, weight, eps):
    """``mx.fast.rms_norm`` over the last axis: x / sqrt(mean(x^2) + eps) * w,
    computed in float32 and returned in x's dtype."""

    x32 = np.asarray(x, np.float32)
    out = x32 / np.sqrt(np.mean(x32 * x32, axis=-1, keepdims=True) + np.float32(eps))
    if weight is not None:
        out = out * np.asarray(weight, np.float32)
    return out.astype(np.asarray(x).dtype)


def silu(x):
    x = np.asarray(x)
    return (x / (1.0 + np.exp(-x))).astype(x.dtype)


def sigmoid(x):
    x = np.asarray(x)
    return (1.0 / (1.0 + np.exp(-x))).astype(x.dtype)


def _ident(x):
    return x


def causal_conv_silu(qkv, conv_state, conv_w, rnd=_ident):
    """``qw/linear_attention.py:61-79``: depthwise cross-correlation of
    ``[conv_state ; qkv]`` (no padding, so L outputs) with weight ``(C, K)``
    (the reference's ``(C, K, 1)`` squeezed), then SiLU. Returns
    ``(silu(out) (L, C), new_tail (K-1, C))``; the tail is taken from the front
    index (``:75-77``), so K=1 keeps nothing.

    ``rnd`` rounds to the activation dtype where the reference materialises
    an array in it: the conv state and weight cast to the input dtype
    (``:69, :72``), the conv output and its SiLU (identity for float32)."""

    qkv = np.asarray(qkv, np.float32)
    w = rnd(np.asarray(conv_w, np.float32).reshape(conv_w.shape[0], -1))
    kernel = w.shape[1]
    conv_in = np.concatenate([rnd(np.asarray(conv_state, np.float32)), qkv], axis=0)
    length = qkv.shape[0]
    out = np.zeros((length, qkv.shape[1]), dtype=np.float64)
    for j in range(kernel):
        out += conv_in[j : j + length].astype(np.float64) * w[None, :, j]
    out = rnd(out.astype(np.float32))
    tail_start = conv_in.shape[0] - (kernel - 1)
    return rnd(silu(out)), conv_in[tail_start:]


def qk_norm(q, k, rnd=_ident):
    """``qw/linear_attention.py:109-113``: q <- Dk^-1 rms_norm(q, eps=1e-6),
    k <- Dk^-1/2 rms_norm(k, eps=1e-6), no weight; eps is hard-coded. ``rnd``
    rounds the rms-norm output and the rescaled value, as the reference
    materialises both."""

    inv_scale = q.shape[-1] ** -0.5
    qn = rnd(np.float32(inv_scale**2) * rnd(rms_norm(q, None, 1e-6)))
    kn = rnd(np.float32(inv_scale) * rnd(rms_norm(k, None, 1e-6)))
    return qn.astype(np.float32), kn.astype(np.float32)


def gated_rms_norm(x, gate, weight, eps, rnd=_ident):
    """``qw/linear_attention.py:22-32``: silu(gate_f32) * rms_norm(x, w, eps)
    in float32, cast back to x's dtype (``rnd``)."""

    normed = rnd(rms_norm(x, weight, eps))
    return rnd(silu(np.asarray(gate, np.float32)) * normed.astype(np.float32))


def split_mixed(mixed, hk, hv, dk, dv):
    """Split the mixed projection row layout ``[q | k | v | z | b | a]``
    (widths Hk*Dk, Hk*Dk, Hv*Dv, Hv*Dv, Hv, Hv) into (qkv, z, b, a): the
    outputs of in_proj_qkv / in_proj_z / in_proj_b / in_proj_a
    (``qw/linear_attention.py:96-101``)."""

    key_dim, value_dim = hk * dk, hv * dv
    conv_dim = 2 * key_dim + value_dim
    qkv = mixed[:, :conv_dim]
    z = mixed[:, conv_dim : conv_dim + value_dim]
    b = mixed[:, conv_dim + value_dim : conv_dim + value_dim + hv]
    a = mixed[:, conv_dim + value_dim + hv : conv_dim + value_dim + 2 * hv]
    return qkv, z, b, a


def block_prologue(mixed, conv_w, conv_state, A_log, dt_bias, hk, hv, dk, dv, rnd=_ident):
    """``qw/linear_attention.py:103-116`` for one sequence: conv + SiLU, q/k/v
    split, q/k norm, log forget gate and beta. Returns float32
    ``(q, k, v, g_log, beta, new_conv_state)`` (values rounded by ``rnd``
    where the reference rounds)."""

    length = mixed.shape[0]
    qkv, _, b, a = split_mixed(np.asarray(mixed, np.float32), hk, hv, dk, dv)
    conv_out, new_conv = causal_conv_silu(qkv, conv_state, conv_w, rnd)
    key_dim = hk * dk
    q = conv_out[:, :key_dim].reshape(length, hk, dk)
    k = conv_out[:, key_dim : 2 * key_dim].reshape(length, hk, dk)
    v = conv_out[:, 2 * key_dim :].reshape(length, hv, dv)
    q, k = qk_norm(q, k, rnd)
    g_log = forget_gate_log(a, A_log, dt_bias)
    beta = rnd(sigmoid(np.asarray(b, np.float32)))
    return q, k, v, g_log, beta, new_conv


def linear_attention_core(
    mixed, conv_w, conv_state, A_log, dt_bias, norm_w, ssm_state, eps, hk, hv, dk, dv,
    scan_dtype=np.float64, rnd=_ident,
):
    """``qw/linear_attention.py:81-124`` from the projections on, for one
    sequence: conv+SiLU (``:103``), q/k/v split (``:104-107``), q/k norm
    (``:109-113``), gates (``:115-116``), scan (``:118-119``), gated RMSNorm
    of ``y`` cast to z's dtype (``:122-124``). ``out_proj`` is not applied.
    ``rnd`` is the activation-dtype rounding (bf16_round for bfloat16).

    Returns ``(out (L, Hv, Dv), new_conv_state, new_ssm_state, y)``."""

    length = mixed.shape[0]
    q, k, v, g_log, beta, new_conv = block_prologue(mixed, conv_w, conv_state, A_log, dt_bias, hk, hv, dk, dv, rnd)
    g = np.exp(g_log.astype(np.float64)) if scan_dtype == np.float64 else np.exp(g_log)
    y, new_ssm = gated_delta_scan(q, k, v, g, beta, ssm_state, scan_dtype)
    _, z, _, _ = split_mixed(np.asarray(mixed, np.float32), hk, hv, dk, dv)
    zr = z.reshape(length, hv, dv)
    out = gated_rms_norm(rnd(y.astype(np.float32)), zr, norm_w, eps, rnd)
    return out, new_conv, new_ssm.astype(np.float32), y


# ---------------------------------------------------------------------------
# Synthetic BASELINE configurations (seeded; value distributions as stated)
# ---------------------------------------------------------------------------


def _l2n(x):
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


def config1_inputs(seed=0):
    """Config 1: fp32, B=1, T=64, Hk=4, Hv=8, Dk=Dv=64. q,k ~ N(0,1) then
    L2-normalised per head; v ~ N(0,1); beta = sigmoid(N); log-decay
    g = -softplus(N); S0 = 0. Returns float32 (q, k, v, g_log, beta, S0)."""

    rng = np.random.default_rng(seed)
    t, hk, hv, d = 64, 4, 8, 64
    q = _l2n(rng.standard_normal((t, hk, d)))
    k = _l2n(rng.standard_normal((t, hk, d)))
    v = rng.standard_normal((t, hv, d))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((t, hv))))
    g_log = -np.logaddexp(0.0, rng.standard_normal((t, hv)))
    s0 = np.zeros((hv, d, d))
    return [a.astype(np.float32) for a in (q, k, v, g_log, beta, s0)]


def decode_inputs(seed, batch, hk, hv, dk, dv, state_std=0.02, with_state=True):
    """Config 2 generator for ONE decode step of ``batch`` sequences:
    q,k ~ N(0,1) L2-normalised, v ~ N(0,1) (all to be rounded to bf16 by the
    caller), beta = sigmoid(N), g_log = -softplus(N), state ~ N(0, state_std)
    float32 ``(B, Hv, Dv, Dk)``."""

    rng = np.random.default_rng(seed)
    q = _l2n(rng.standard_normal((batch, hk, dk))).astype(np.float32)
    k = _l2n(rng.standard_normal((batch, hk, dk))).astype(np.float32)
    v = rng.standard_normal((batch, hv, dv)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((batch, hv))))).astype(np.float32)
    g_log = (-np.logaddexp(0.0, rng.standard_normal((batch, hv)))).astype(np.float32)
    state = None
    if with_state:
        state = (rng.standard_normal((batch, hv, dv, dk), dtype=np.float32) * state_std)
    return q, k, v, g_log, beta, state


def prefill_inputs(seed, total, hk, hv, dk, dv):
    """Configs 3 and 5 per-token draws: q,k ~ N(0,1) L2-normalised,
    v ~ N(0,1), beta = sigmoid(N), g_log = -softplus(N); float32 arrays of
    ``total`` packed tokens (to be rounded to bf16 by the caller for q/k/v)."""

    rng = np.random.default_rng(seed)
    q = _l2n(rng.standard_normal((total, hk, dk), dtype=np.float32))
    k = _l2n(rng.standard_normal((total, hk, dk), dtype=np.float32))
    v = rng.standard_normal((total, hv, dv), dtype=np.float32)
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((total, hv), dtype=np.float32)))
    g_log = -np.logaddexp(np.float32(0.0), rng.standard_normal((total, hv), dtype=np.float32))
    return q, k, v, g_log.astype(np.float32), beta.astype(np.float32)


def config5_lengths(n_seq=64, lo=256, hi=16384, seed=1):
    """Config 5 sequence lengths: ``default_rng(1).integers(256, 16384,
    size=64, endpoint=True)``."""

    return np.random.default_rng(seed).integers(lo, hi, size=n_seq, endpoint=True)


def block_inputs(seed, batch, length, hk=16, hv=32, dk=128, dv=128, kernel=4):
    """Config 4 generator: mixed projection ``(B*T, 2HkDk + 2HvDv + 2Hv)``
    ~ N(0,1) (rounded to bf16 by the caller), conv_w ~ N(0, 0.1) ``(C, K)``,
    A_log ~ U(0, 1.5), dt_bias ~ N(0, 0.1), norm_w = 1."""

    rng = np.random.default_rng(seed)
    width = 2 * hk * dk + 2 * hv * dv + 2 * hv
    conv_dim = 2 * hk * dk + hv * dv
    mixed = rng.standard_normal((batch * length, width), dtype=np.float32)
    conv_w = (rng.standard_normal((conv_dim, kernel), dtype=np.float32) * 0.1)
    A_log = rng.uniform(0.0, 1.5, size=hv).astype(np.float32)
    dt_bias = (rng.standard_normal(hv) * 0.1).astype(np.float32)
    norm_w = np.ones(dv, np.float32)
    return mixed, conv_w, A_log, dt_bias, norm_w


def bf16_round(x):
    """Round float32 to the nearest bfloat16 (ties to even), returned as
    float32: the values a bf16 tensor holds."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def rel_l2(actual, expected):
    """||actual - expected||_2 / ||expected||_2 in float64 (0 if both are 0)."""

    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    den = math.sqrt(float(np.sum(e * e)))
    num = math.sqrt(float(np.sum((a - e) ** 2)))
    return num / den if den > 0 else num


# ---------------------------------------------------------------------------
# Affine-quantized linear projections (model/moe_block.py:23-50).
#
# The reference calls mx.quantized_matmul (mlx 0.32.2, uv.lock:268-269), a
# third-party kernel absent from the reference tree.  Its published affine
# format: the unsigned `bits`-bit values of a row are packed into uint32
# words along the input dimension, value j of a word in bits
# [j * bits, (j + 1) * bits); one scale and one bias per `group_size`
# consecutive inputs; W = scale * q + bias.  Parity for this part is unpinned
# against mlx itself (not installable here): the checks are the format's
# known-answer packings and this restatement.


def pack_affine(q, bits):
    """Pack unsigned values q[n, k] (< 2**bits) into uint32 words [n, k * bits / 32]."""

    q = np.asarray(q, np.uint64)
    n, k = q.shape
    per = 32 // bits
    if 32 % bits or k % per:
        raise ValueError("k must fill whole words")
    if np.any(q >> np.uint64(bits)):
        raise ValueError("value out of range for the bit width")
    q = q.reshape(n, k // per, per)
    shifts = (np.arange(per, dtype=np.uint64) * np.uint64(bits))[None, None, :]
    return np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)


def unpack_affine(w, bits):
    """The inverse of pack_affine: uint32 words [n, kw] -> values [n, kw * 32 / bits]."""

    w = np.asarray(w, np.uint32).astype(np.uint64)
    n, kw = w.shape
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint64) * np.uint64(bits))[None, None, :]
    vals = (w[:, :, None] >> shifts) & np.uint64((1 << bits) - 1)
    return vals.reshape(n, kw * per).astype(np.int64)


def quantize_affine(dense, bits, group_size):
    """Test weights: per-group min/max affine quantization of dense[n, k] with
    bf16 scales and biases (bias = the group minimum, scale = range / levels).
    Returns (words, scales, biases) with scales and biases as float32 holding
    bf16 values."""

    dense = np.asarray(dense, np.float32)
    n, k = dense.shape
    g = dense.reshape(n, k // group_size, group_size)
    lo, hi = g.min(axis=2), g.max(axis=2)
    levels = (1 << bits) - 1
    scales = bf16_round(np.maximum(hi - lo, 1e-8) / levels)
    biases = bf16_round(lo)
    q = np.rint((g - biases[:, :, None]) / scales[:, :, None])
    q = np.clip(q, 0, levels).astype(np.int64).reshape(n, k)
    return pack_affine(q, bits), scales, biases


def dequant_affine(words, scales, biases, bits, group_size):
    """W[n, k] = scale * q + bias, each element rounded once to bf16 (the
    operand the tensor-core GEMM multiplies).  scale * q is exact in float32
    (an 8-bit mantissa times an integer below 256), so the float32 sum is one
    fused multiply-add.  biases=None means zero."""

    q = unpack_affine(words, bits).astype(np.float32)
    n, k = q.shape
    s = np.repeat(np.asarray(scales, np.float32), group_size, axis=1)
    b = np.zeros_like(s) if biases is None else np.repeat(np.asarray(biases, np.float32), group_size, axis=1)
    if s.shape != (n, k):
        raise ValueError("scales do not match the packed weights")
    return bf16_round(s * q + b)


def quantized_linear_ref(x, words, scales, biases, bits, group_size):
    """x[m, k] @ W^T in float64 with W from dequant_affine; returns float64 [m, n]."""

    w = dequant_affine(words, scales, biases, bits, group_size).astype(np.float64)
    return np.asarray(x, np.float64) @ w.T


# ---------------------------------------------------------------------------
# Softmax attention layer (qw/attention.py:40-99) with its growing KV cache
# (cache/kv_cache.py:28-102): grouped-query heads, the output gate carried in
# q_proj's second half, q/k RMS norms with weights, rotary embedding of the
# leading rotary_dim features (model/rope.py: feature i pairs with
# i + rotary_dim / 2), the causal mask aligned to the newest query.
# ---------------------------------------------------------------------------


def rope_leading(x, rotary_dim, base, offset):
    """x (L, H, D): rotate features [0, rotary_dim) of the token at position
    offset + l by angle (offset + l) * base ** (-2 i / rotary_dim)."""

    x = np.asarray(x, np.float64)
    out = x.copy()
    half = rotary_dim // 2
    inv = base ** (-np.arange(half, dtype=np.float64) * 2.0 / rotary_dim)
    ang = (offset + np.arange(x.shape[0], dtype=np.float64))[:, None] * inv[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half], x[..., half:rotary_dim]
    out[..., :half] = a * cos - b * sin
    out[..., half:rotary_dim] = b * cos + a * sin
    return out


def attention_core(q, keys, values, scale):
    """q (L, H, D) for the newest L of T cached positions; keys/values
    (Hkv, T, D). Query l of head h sees key positions <= T - L + l of head
    h // (H / Hkv). Returns (L, H, D) in float64."""

    q = np.asarray(q, np.float64)
    keys = np.asarray(keys, np.float64)
    values = np.asarray(values, np.float64)
    length, heads, _ = q.shape
    hkv, t, _ = keys.shape
    rep = heads // hkv
    out = np.empty_like(q)
    allowed = np.arange(t)[None, :] <= (t - length + np.arange(length))[:, None]
    for h in range(heads):
        s = q[:, h, :] @ keys[h // rep].T * scale
        s = np.where(allowed, s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[:, h, :] = (p / p.sum(axis=1, keepdims=True)) @ values[h // rep]
    return out


def attention_layer(x, w, keys, values, heads, kv_heads, head_dim, rotary_dim, theta, eps, rnd=_ident):
    """One call of ``Qwen3_5Attention.__call__`` (qw/attention.py:40-99):
    x (L, hidden) float; dense projections w[q_proj|k_proj|v_proj|o_proj]
    (out, in) and the norm weights; keys/values the cache (Hkv, T0, D) before
    the call. ``rnd`` rounds where the reference materializes activations in
    a narrower dtype. Returns (out (L, hidden), keys, values) with the cache
    grown by L."""

    x = np.asarray(x, np.float64)
    length = x.shape[0]
    qg = rnd(x @ np.asarray(w["q_proj"], np.float64).T).reshape(length, heads, 2 * head_dim)  # :56-59
    q, gate = qg[..., :head_dim], qg[..., head_dim:]
    q = rnd(rms_norm(q, w["q_norm"], eps))  # :60
    k = rnd(rms_norm(rnd(x @ np.asarray(w["k_proj"], np.float64).T).reshape(length, kv_heads, head_dim),
                     w["k_norm"], eps))  # :62-65
    v = rnd(x @ np.asarray(w["v_proj"], np.float64).T).reshape(length, kv_heads, head_dim)  # :66-68
    offset = keys.shape[1]  # :74
    q = rnd(rope_leading(q, rotary_dim, theta, offset))  # :78-80
    k = rnd(rope_leading(k, rotary_dim, theta, offset))  # :81-83
    keys = np.concatenate([keys, k.transpose(1, 0, 2)], axis=1)  # :85
    values = np.concatenate([values, v.transpose(1, 0, 2)], axis=1)
    o = rnd(attention_core(q, keys, values, head_dim ** -0.5)).reshape(length, heads * head_dim)  # :87-94
    o = rnd(o * rnd(sigmoid(gate.reshape(length, heads * head_dim))))  # :96
    out = rnd(o @ np.asarray(w["o_proj"], np.float64).T)  # :97
    return out, keys, values
