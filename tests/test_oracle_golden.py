"""The oracle against the golden vectors produced by the reference's own code
(``tests/golden/make_golden.py``). CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from make_golden import ATTN, GDN_CASES, LAYER, METAL_SHAPES, LONG_LENGTH, attn_case, layer_case, metal_key, sha
from oracle import gdn_oracle as O
from oracle import oracle_c


@pytest.mark.parametrize("shape", METAL_SHAPES)
def test_metal_generator_reproduces_reference_inputs(shape, manifest):
    inputs = O.metal_test_inputs(*shape)
    assert [sha(a) for a in inputs] == manifest["inputs"][metal_key(shape)]


def _check_state(golden, key, state, rtol, atol, sum_rtol=1e-9):
    if f"{key}/state" in golden:
        np.testing.assert_allclose(state, golden[f"{key}/state"], rtol=rtol, atol=atol)
    else:
        np.testing.assert_allclose(state[::4], golden[f"{key}/state_heads_every4"], rtol=rtol, atol=atol)
        np.testing.assert_allclose(state.sum(), golden[f"{key}/state_sum"], rtol=sum_rtol, atol=1e-9)
        np.testing.assert_allclose((state.astype(np.float64) ** 2).sum(), golden[f"{key}/state_sumsq"], rtol=sum_rtol)


@pytest.mark.parametrize("shape", METAL_SHAPES)
def test_numpy_oracle_matches_reference_float64_recurrence(shape, golden):
    key = metal_key(shape)
    inputs = O.metal_test_inputs(*shape)
    y, state = O.gated_delta_scan(*inputs)
    np.testing.assert_allclose(y, golden[f"{key}/y"], rtol=1e-6, atol=1e-7)
    _check_state(golden, key, state, 1e-6, 1e-7)
    # reference_f64 is the restated test recurrence itself
    y2, s2 = O.reference_f64(inputs)
    np.testing.assert_allclose(y2, y, rtol=1e-12, atol=1e-13)


@pytest.mark.parametrize("shape", METAL_SHAPES)
def test_c_oracle_matches_reference_float64_recurrence(shape, golden):
    key = metal_key(shape)
    q, k, v, g, beta, state = O.metal_test_inputs(*shape)
    cu = np.array([0, q.shape[0]])
    y, st = oracle_c.scan_varlen(q, k, v, g, beta, cu, state[None])
    np.testing.assert_allclose(y, golden[f"{key}/y"], rtol=2e-6, atol=2e-7)
    _check_state(golden, key, st[0].astype(np.float64), 2e-6, 2e-7, sum_rtol=1e-6)


def test_long_scan_golden(golden, manifest):
    inputs = O.metal_test_inputs(LONG_LENGTH)
    assert [sha(a) for a in inputs] == manifest["inputs"]["long"]
    q, k, v, g, beta, state = inputs
    y, st = oracle_c.scan_varlen(q, k, v, g, beta, np.array([0, LONG_LENGTH]), state[None])
    np.testing.assert_allclose(y[::8], golden["long/y_every8"], rtol=2e-6, atol=2e-7)
    np.testing.assert_allclose(st[0], golden["long/state"], rtol=2e-6, atol=2e-7)


def test_varlen_oracle_equals_per_sequence_calls():
    rng = np.random.default_rng(5)
    cu = np.array([0, 3, 3, 10, 11])
    n, hk, hv, dk, dv = 11, 2, 4, 16, 8
    q = rng.standard_normal((n, hk, dk)).astype(np.float32)
    k = O._l2n(rng.standard_normal((n, hk, dk))).astype(np.float32)
    v = rng.standard_normal((n, hv, dv)).astype(np.float32)
    g = rng.uniform(0.5, 1, (n, hv)).astype(np.float32)
    beta = rng.uniform(0, 1, (n, hv)).astype(np.float32)
    states = rng.standard_normal((4, hv, dv, dk)).astype(np.float32)
    y, st = O.scan_varlen(q, k, v, g, beta, cu, states)
    yc, stc = oracle_c.scan_varlen(q, k, v, g, beta, cu, states)
    np.testing.assert_allclose(yc, y, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(stc, st, rtol=2e-6, atol=2e-6)
    np.testing.assert_array_equal(st[1], states[1])  # empty sequence keeps its state


@pytest.mark.parametrize("seed,seq_len", GDN_CASES)
def test_gates_and_scan_match_reference_ops_path(seed, seq_len, golden, manifest):
    key = f"gdn_{seed}_{seq_len}"
    x = O.gdn_test_inputs(seed, seq_len)
    assert {k: sha(v) for k, v in x.items()} == manifest["inputs"][key]
    g = O.forget_gate(x["a"], x["A_log"], x["dt_bias"])
    beta = O.sigmoid(x["b"])
    np.testing.assert_allclose(g, golden[f"{key}/g"], rtol=1e-6, atol=0)
    np.testing.assert_allclose(beta, golden[f"{key}/beta"], rtol=1e-6, atol=0)
    assert np.all(g > 0) and np.all(g <= 1)
    y, st = O.gated_delta_scan(x["q"], x["k"], x["v"], g, beta, np.zeros((6, 8, 16), np.float32), np.float32)
    np.testing.assert_allclose(y, golden[f"{key}/y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st, golden[f"{key}/state"], rtol=1e-5, atol=1e-6)
    # log-decay form is the log of the multiplier
    np.testing.assert_allclose(np.exp(O.forget_gate_log(x["a"], x["A_log"], x["dt_bias"])), g, rtol=1e-6)


def _layer_forward(w, x, conv_state, ssm_state):
    """Projections (dense, as the golden run used) around the oracle core."""
    hk, hv, dk, dv = LAYER["hk"], LAYER["hv"], LAYER["dk"], LAYER["dv"]
    mixed = np.concatenate(
        [x @ w["in_proj_qkv"].T, x @ w["in_proj_z"].T, x @ w["in_proj_b"].T, x @ w["in_proj_a"].T], axis=1
    ).astype(np.float32)
    out, conv, ssm, _ = O.linear_attention_core(
        mixed, w["conv1d_weight"][:, :, 0], conv_state, w["A_log"], w["dt_bias"], w["norm_weight"],
        ssm_state, LAYER["eps"], hk, hv, dk, dv, scan_dtype=np.float32,
    )
    return out.reshape(x.shape[0], -1) @ w["out_proj"].T, conv, ssm


def _fresh():
    conv_dim = 2 * LAYER["hk"] * LAYER["dk"] + LAYER["hv"] * LAYER["dv"]
    return (np.zeros((LAYER["kernel"] - 1, conv_dim), np.float32),
            np.zeros((LAYER["hv"], LAYER["dv"], LAYER["dk"]), np.float32))


@pytest.mark.parametrize("seq_len", [1, 6])
def test_layer_core_matches_reference_layer(seq_len, golden, manifest):
    key = f"layer_fresh_{seq_len}"
    w, x = layer_case(0, 100, seq_len)
    assert {k: sha(v) for k, v in {**w, "x": x}.items()} == manifest["inputs"][key]
    out, conv, ssm = _layer_forward(w, x, *_fresh())
    np.testing.assert_allclose(out, golden[f"{key}/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(conv, golden[f"{key}/conv_state"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ssm, golden[f"{key}/ssm_state"], rtol=1e-5, atol=1e-6)


def test_layer_core_stepwise_and_chunked_carry_both_states(golden):
    w, x = layer_case(1, 101, 5)
    conv, ssm = _fresh()
    outs = []
    for t in range(5):
        o, conv, ssm = _layer_forward(w, x[t : t + 1], conv, ssm)
        outs.append(o[0])
    np.testing.assert_allclose(np.stack(outs), golden["layer_steps/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(conv, golden["layer_steps/conv_state"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ssm, golden["layer_steps/ssm_state"], rtol=1e-5, atol=1e-6)

    w, _ = layer_case(2, 102, 1)
    rng = np.random.default_rng(102)
    xs = [rng.standard_normal((3, LAYER["hidden"])).astype(np.float32) for _ in range(4)]
    conv, ssm = _fresh()
    outs = []
    for xc in xs:
        o, conv, ssm = _layer_forward(w, xc, conv, ssm)
        outs.append(o)
    np.testing.assert_allclose(np.concatenate(outs), golden["layer_chunks/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(conv, golden["layer_chunks/conv_state"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ssm, golden["layer_chunks/ssm_state"], rtol=1e-5, atol=1e-6)


def test_bf16_round_is_round_to_nearest_even():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 10
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.bf16_round(x), want)


def _attn(x, w, keys, values):
    return O.attention_layer(x, w, keys, values, ATTN["heads"], ATTN["kv_heads"], ATTN["head_dim"],
                             ATTN["rotary"], ATTN["theta"], ATTN["eps"])


def _empty_cache():
    return np.zeros((ATTN["kv_heads"], 0, ATTN["head_dim"])), np.zeros((ATTN["kv_heads"], 0, ATTN["head_dim"]))


@pytest.mark.parametrize("seq_len", [1, 6])
def test_attention_oracle_matches_reference_layer(seq_len, golden, manifest):
    w = attn_case(0)
    x = np.random.default_rng(200).standard_normal((seq_len, ATTN["hidden"])).astype(np.float32)
    assert manifest["inputs"][f"attn_fresh_{seq_len}"]["x"] == sha(x)
    assert manifest["inputs"][f"attn_fresh_{seq_len}"]["q_proj"] == sha(w["q_proj"])
    out, keys, values = _attn(x, w, *_empty_cache())
    np.testing.assert_allclose(out, golden[f"attn_fresh_{seq_len}/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(keys, golden[f"attn_fresh_{seq_len}/keys"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(values, golden[f"attn_fresh_{seq_len}/values"], rtol=1e-5, atol=1e-6)


def test_attention_oracle_decode_steps_and_offset_chunks(golden):
    w = attn_case(1)
    x = np.random.default_rng(201).standard_normal((5, ATTN["hidden"])).astype(np.float32)
    keys, values = _empty_cache()
    outs = []
    for t in range(5):
        o, keys, values = _attn(x[t:t + 1], w, keys, values)
        outs.append(o[0])
    np.testing.assert_allclose(np.stack(outs), golden["attn_steps/out"], rtol=1e-4, atol=1e-5)
    batched, _, _ = _attn(x, w, *_empty_cache())
    np.testing.assert_allclose(batched, golden["attn_steps/batched"], rtol=1e-4, atol=1e-5)

    w = attn_case(3)
    xs = np.random.default_rng(203).standard_normal((3, 4, ATTN["hidden"])).astype(np.float32)
    keys, values = _empty_cache()
    outs = []
    for xc in xs:
        o, keys, values = _attn(xc, w, keys, values)
        outs.append(o)
    np.testing.assert_allclose(np.concatenate(outs), golden["attn_chunks/out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(keys, golden["attn_chunks/keys"], rtol=1e-5, atol=1e-6)


def test_rope_leaves_the_tail_and_rotates_pairs():
    # the reference's rope test: features past rotary_dim pass unchanged
    x = np.random.default_rng(1).standard_normal((3, 2, 16))
    out = O.rope_leading(x, 4, 10000.0, 7)
    np.testing.assert_array_equal(out[..., 4:], x[..., 4:])
    # position 0 is the identity; a pair keeps its norm
    np.testing.assert_allclose(O.rope_leading(x, 4, 10000.0, 0)[0], x[0])
    np.testing.assert_allclose(np.hypot(out[..., 0], out[..., 2]), np.hypot(x[..., 0], x[..., 2]))
