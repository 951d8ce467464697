"""The fused linear-attention block (gdn_fused_block) against the reference's
own layer (golden vectors, float32) and against the oracle's bfloat16
restatement (rounding where the reference materialises bf16 arrays)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200.linear_attention import LinearAttentionShape
from gpu_helpers import dev, n, t
from make_golden import LAYER, layer_case
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

SHAPE = LinearAttentionShape(LAYER["hk"], LAYER["hv"], LAYER["dk"], LAYER["dv"], LAYER["kernel"])


def _layer(w):
    return gdn_b200.Qwen3_5LinearAttention(
        SHAPE, LAYER["eps"], t(w["in_proj_qkv"]), t(w["in_proj_z"]), t(w["in_proj_a"]), t(w["in_proj_b"]),
        t(w["conv1d_weight"]), t(w["A_log"]), t(w["dt_bias"]), t(w["norm_weight"]), t(w["out_proj"]),
    )


def _cache():
    return gdn_b200.RecurrentCache(LAYER["kernel"], SHAPE.conv_dim, LAYER["hv"], LAYER["dv"], LAYER["dk"],
                                   device=dev())


@pytest.mark.parametrize("seq_len", [1, 6])
def test_layer_matches_reference_layer(seq_len, golden):
    # tf32 would round the projections: this comparison is float32
    torch.backends.cuda.matmul.allow_tf32 = False
    key = f"layer_fresh_{seq_len}"
    w, x = layer_case(0, 100, seq_len)
    cache = _cache()
    out = _layer(w)(t(x), cache)
    np.testing.assert_allclose(n(out), golden[f"{key}/out"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(n(cache.conv_state), golden[f"{key}/conv_state"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n(cache.ssm_state), golden[f"{key}/ssm_state"], rtol=1e-4, atol=1e-5)
    assert cache.size == seq_len


def test_layer_stepwise_and_chunked_calls_carry_both_states(golden):
    torch.backends.cuda.matmul.allow_tf32 = False
    w, x = layer_case(1, 101, 5)
    layer, cache = _layer(w), _cache()
    stepwise = torch.stack([layer(t(x[i]), cache) for i in range(5)])
    np.testing.assert_allclose(n(stepwise), golden["layer_steps/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(n(cache.conv_state), golden["layer_steps/conv_state"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n(cache.ssm_state), golden["layer_steps/ssm_state"], rtol=1e-4, atol=1e-5)
    assert cache.size == 5
    batched = layer(t(x), _cache())
    torch.testing.assert_close(batched, stepwise, rtol=1e-4, atol=1e-5)

    w, _ = layer_case(2, 102, 1)
    rng = np.random.default_rng(102)
    xs = [rng.standard_normal((3, LAYER["hidden"])).astype(np.float32) for _ in range(4)]
    layer, cache = _layer(w), _cache()
    outs = [layer(t(xc), cache) for xc in xs]
    np.testing.assert_allclose(n(torch.cat(outs)), golden["layer_chunks/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(n(cache.ssm_state), golden["layer_chunks/ssm_state"], rtol=1e-4, atol=1e-5)
    shapes = {(tuple(cache.conv_state.shape), tuple(cache.ssm_state.shape))}
    assert len(shapes) == 1 and cache.size == 12


def _bf16_block_case(lengths, hk, hv, dk, dv, seed, algo="auto", kernel=4, conv_dtype=torch.bfloat16):
    B = len(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    N = int(cu[-1])
    shape = LinearAttentionShape(hk, hv, dk, dv, kernel)
    rng = np.random.default_rng(seed)
    mixed = O.bf16_round(rng.standard_normal((N, shape.mixed_width)).astype(np.float32))
    conv_w = (rng.standard_normal((shape.conv_dim, kernel)) * 0.1).astype(np.float32)
    A_log = rng.uniform(0, 1.5, hv).astype(np.float32)
    dt_bias = (rng.standard_normal(hv) * 0.1).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    conv_state = O.bf16_round((rng.standard_normal((B, kernel - 1, shape.conv_dim))).astype(np.float32))
    ssm = (rng.standard_normal((B, hv, dv, dk)) * 0.02).astype(np.float32)
    eps = 1e-6

    cs, ss = t(conv_state, conv_dtype), t(ssm)
    out, _, _ = gdn_b200.gated_delta_block(
        t(mixed, torch.bfloat16), shape, t(conv_w), t(A_log), t(dt_bias), t(norm_w), eps, cs, ss,
        cu_seqlens=t(cu, torch.int64), algo=algo,
    )
    got_out, got_conv, got_ssm = n(out), n(cs), n(ss)
    exp_out, exp_conv, exp_ssm = [], [], []
    for b in range(B):
        if lengths[b] == 0:  # an empty sequence keeps both states
            exp_conv.append(conv_state[b])
            exp_ssm.append(ssm[b])
            continue
        o, c, s, _ = O.linear_attention_core(
            mixed[cu[b] : cu[b + 1]], conv_w, conv_state[b], A_log, dt_bias, norm_w, ssm[b], eps,
            hk, hv, dk, dv, rnd=O.bf16_round,
        )
        exp_out.append(o)
        exp_conv.append(c)
        exp_ssm.append(s)
    return got_out, np.concatenate(exp_out), got_conv, np.stack(exp_conv), got_ssm, np.stack(exp_ssm)


@pytest.mark.parametrize("lengths", [[37, 90], [1, 2, 0, 5], [130]])
def test_bf16_block_matches_oracle(lengths):
    go, eo, gc, ec, gs, es = _bf16_block_case(lengths, 2, 4, 64, 32, seed=len(lengths))
    assert O.rel_l2(go, eo) < 2e-3
    assert O.rel_l2(gs, es) < 2e-3
    np.testing.assert_array_equal(gc, ec)  # the conv tail is a copy of bf16 values


def test_bf16_block_at_model_head_shape():
    go, eo, gc, ec, gs, es = _bf16_block_case([96, 160], 16, 32, 128, 128, seed=4)
    assert O.rel_l2(go, eo) < 2e-3
    assert O.rel_l2(gs, es) < 2e-3
    np.testing.assert_array_equal(gc, ec)


@pytest.mark.parametrize("kernel", [1, 2, 3])
def test_bf16_block_other_conv_widths(kernel):
    go, eo, gc, ec, gs, es = _bf16_block_case([5, 70], 2, 4, 32, 64, seed=10 + kernel, kernel=kernel)
    assert O.rel_l2(go, eo) < 2e-3
    assert O.rel_l2(gs, es) < 2e-3
    if kernel > 1:
        np.testing.assert_array_equal(gc, ec)


def test_bf16_block_general_head_dims():
    """Head dims that are not powers of two take the general prologue and
    epilogue kernels and the serial scan."""
    go, eo, gc, ec, gs, es = _bf16_block_case([33, 2], 3, 6, 48, 40, seed=21)
    assert O.rel_l2(go, eo) < 2e-3
    assert O.rel_l2(gs, es) < 2e-3
    np.testing.assert_array_equal(gc, ec)


@pytest.mark.parametrize("kernel", [1, 2, 3, 4])
@pytest.mark.parametrize("conv_dtype", [torch.bfloat16, torch.float32])
def test_bf16_chunked_block_edges(kernel, conv_dtype):
    """The chunked block at 128-dim heads, two value heads per key head:
    sequences of 0, 1 and 5 tokens (ragged single chunks), one whose second
    chunk starts on its conv history, each conv width and both conv-state
    dtypes."""
    go, eo, gc, ec, gs, es = _bf16_block_case([5, 70, 1, 0, 200], 4, 8, 128, 128, seed=30 + kernel, algo="chunked",
                                              kernel=kernel, conv_dtype=conv_dtype)
    assert O.rel_l2(go, eo) < 2e-3
    assert O.rel_l2(gs, es) < 2e-3
    if kernel > 1:
        np.testing.assert_array_equal(gc, ec)
