"""The CUDA scan through the reference-shaped API against the reference's
own known answers (golden vectors) and the oracle: the Metal kernel's test
shapes contiguous and strided, the long prefill-then-decode split, dtype
behaviour, gates, and the step/scan identities. Tolerances are the
reference's (rtol 2e-5, atol 2e-6 for float32)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gpu_helpers import n, t
from make_golden import GDN_CASES, LONG_LENGTH, METAL_SHAPES, metal_key
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-5, 2e-6


def _check_state(golden, key, state):
    if f"{key}/state" in golden:
        np.testing.assert_allclose(state, golden[f"{key}/state"], rtol=RTOL, atol=ATOL)
    else:
        np.testing.assert_allclose(state[::4], golden[f"{key}/state_heads_every4"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("shape", METAL_SHAPES)
@pytest.mark.parametrize("strided", [False, True])
def test_scan_matches_reference_known_answers_and_keeps_input_state(shape, strided, golden):
    inputs = [t(a) for a in O.metal_test_inputs(*shape)]
    if strided:  # innermost stride 2, as tests/test_gated_delta_metal.py:51-52
        inputs = [torch.stack([a, a], dim=-1)[..., 0] for a in inputs]
    before = inputs[-1].clone()
    y, state = gdn_b200.gated_delta_scan(*inputs)
    assert y.dtype == state.dtype == torch.float32
    key = metal_key(shape)
    np.testing.assert_allclose(n(y), golden[f"{key}/y"], rtol=RTOL, atol=ATOL)
    _check_state(golden, key, n(state))
    assert torch.equal(inputs[-1], before)


def test_token_and_head_strided_views_are_read_in_place():
    q, k, v, g, beta, s0 = O.metal_test_inputs(33, 64, 32, 2, 4)
    big = t(np.concatenate([q, k], axis=1))  # (L, 4, Dk): q heads then k heads
    qv, kv = big[:, :2], big[:, 2:]
    assert not qv.is_contiguous() and qv.stride(-1) == 1
    y, st = gdn_b200.gated_delta_scan(qv, kv, t(v), t(g), t(beta), t(s0))
    ey, est = O.gated_delta_scan(q, k, v, g, beta, s0)
    np.testing.assert_allclose(n(y), ey, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(n(st), est, rtol=RTOL, atol=ATOL)


def test_long_scan_and_prefill_then_decode_preserve_carried_state(golden):
    inputs = [t(a) for a in O.metal_test_inputs(LONG_LENGTH)]
    whole_y, whole_state = gdn_b200.gated_delta_scan(*inputs)
    state = inputs[-1]
    outputs = []
    bounds = [0, 1, 128, 383, 1024, 1920, *range(1921, 2049)]
    for start, end in zip(bounds, bounds[1:]):
        y, state = gdn_b200.gated_delta_scan(*(a[start:end] for a in inputs[:-1]), state)
        outputs.append(y)
    split_y = torch.cat(outputs)
    for actual in (whole_y, split_y):
        np.testing.assert_allclose(n(actual)[::8], golden["long/y_every8"], rtol=RTOL, atol=ATOL)
    for actual in (whole_state, state):
        np.testing.assert_allclose(n(actual), golden["long/state"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("case", ["float16", "bfloat16", "mixed", "small_head"])
def test_other_dtypes_follow_reference_promotion(case):
    arrays = O.metal_test_inputs(5, key_dim=16 if case == "small_head" else 128)
    inputs = [t(a) for a in arrays]
    if case in ("float16", "bfloat16"):
        inputs = [a.to(getattr(torch, case)) for a in inputs]
    elif case == "mixed":
        inputs[2] = inputs[2].half()
    y, state = gdn_b200.gated_delta_scan(*inputs)
    want = torch.float32 if case in ("mixed", "small_head") else getattr(torch, case)
    assert y.dtype == state.dtype == want
    ey, est = O.gated_delta_scan(*[n(a) for a in inputs])
    tol = 2e-5 if want == torch.float32 else 1e-2
    assert O.rel_l2(n(y), ey) < tol
    assert O.rel_l2(n(state), est) < tol


@pytest.mark.parametrize("seed,seq_len", GDN_CASES)
def test_device_gates_and_scan_match_reference_ops_path(seed, seq_len, golden):
    key = f"gdn_{seed}_{seq_len}"
    x = {k: t(v) for k, v in O.gdn_test_inputs(seed, seq_len).items()}
    g = gdn_b200.forget_gate(x["a"], x["A_log"], x["dt_bias"])
    np.testing.assert_allclose(n(g), golden[f"{key}/g"], rtol=1e-5, atol=1e-7)
    assert bool((g > 0).all()) and bool((g <= 1).all())
    lg = gdn_b200.forget_gate(x["a"], x["A_log"], x["dt_bias"], log=True)
    np.testing.assert_allclose(np.exp(n(lg)), golden[f"{key}/g"], rtol=1e-5, atol=1e-7)
    beta = torch.sigmoid(x["b"])
    y, st = gdn_b200.gated_delta_scan(x["q"], x["k"], x["v"], g, beta, torch.zeros(6, 8, 16, device=g.device))
    np.testing.assert_allclose(n(y), golden[f"{key}/y"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(n(st), golden[f"{key}/state"], rtol=1e-4, atol=1e-5)


def test_scan_continues_from_a_carried_state():
    x = {k: t(v) for k, v in O.gdn_test_inputs(1, 5).items()}
    g, beta = gdn_b200.forget_gate(x["a"], x["A_log"], x["dt_bias"]), torch.sigmoid(x["b"])
    zero = torch.zeros(6, 8, 16, device=g.device)
    wy, ws = gdn_b200.gated_delta_scan(x["q"], x["k"], x["v"], g, beta, zero)
    y1, mid = gdn_b200.gated_delta_scan(x["q"][:2], x["k"][:2], x["v"][:2], g[:2], beta[:2], zero)
    y2, fin = gdn_b200.gated_delta_scan(x["q"][2:], x["k"][2:], x["v"][2:], g[2:], beta[2:], mid)
    torch.testing.assert_close(torch.cat([y1, y2]), wy, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(fin, ws, rtol=1e-5, atol=1e-6)


def test_single_step_matches_the_scan_of_one():
    x = {k: t(v) for k, v in O.gdn_test_inputs(2, 1).items()}
    g, beta = gdn_b200.forget_gate(x["a"], x["A_log"], x["dt_bias"]), torch.sigmoid(x["b"])
    state = torch.zeros(6, 8, 16, device=g.device)
    sy, ss = gdn_b200.gated_delta_scan(x["q"], x["k"], x["v"], g, beta, state)
    q = torch.repeat_interleave(x["q"][0], 3, dim=0)
    k = torch.repeat_interleave(x["k"][0], 3, dim=0)
    ty, ts = gdn_b200.gated_delta_step(q, k, x["v"][0], g[0], beta[0], state)
    torch.testing.assert_close(ty, sy[0], rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(ts, ss, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("invalid", ["k", "v", "g", "beta", "state", "heads", "empty"])
def test_invalid_shapes_on_device_are_rejected_before_launch(invalid):
    inputs = [t(a) for a in O.metal_test_inputs(5)]
    index = {"k": 1, "v": 2, "g": 3, "beta": 4, "state": 5}
    if invalid in index:
        inputs[index[invalid]] = inputs[index[invalid]][:1]
    elif invalid == "heads":
        inputs[0] = inputs[0][:, :1].repeat(1, 3, 1)
        inputs[1] = inputs[0]
    else:
        inputs = [a[:0] for a in inputs[:-1]] + inputs[-1:]
    with pytest.raises(ValueError):
        gdn_b200.gated_delta_scan(*inputs)


def test_varlen_serial_scan_with_empty_and_ragged_sequences():
    from oracle import oracle_c

    rng = np.random.default_rng(11)
    lengths = [0, 1, 37, 0, 64, 5]
    cu = np.concatenate([[0], np.cumsum(lengths)])
    N, hk, hv, dk, dv = int(cu[-1]), 3, 6, 32, 5
    q = O._l2n(rng.standard_normal((N, hk, dk))).astype(np.float32)
    k = O._l2n(rng.standard_normal((N, hk, dk))).astype(np.float32)
    v = rng.standard_normal((N, hv, dv)).astype(np.float32)
    g = rng.uniform(0.9, 1, (N, hv)).astype(np.float32)
    beta = rng.uniform(0, 1, (N, hv)).astype(np.float32)
    s0 = (rng.standard_normal((len(lengths), hv, dv, dk)) * 0.1).astype(np.float32)
    y, st = gdn_b200.gated_delta_scan_varlen(t(q), t(k), t(v), t(g), t(beta), t(s0), t(cu, torch.int64),
                                             algo="serial")
    ey, est = oracle_c.scan_varlen(q, k, v, g, beta, cu, s0)
    np.testing.assert_allclose(n(y), ey, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(n(st), est, rtol=RTOL, atol=ATOL)
    np.testing.assert_array_equal(n(st)[0], s0[0])
    # in place: state_out is the input state
    s_dev = t(s0)
    gdn_b200.gated_delta_scan_varlen(t(q), t(k), t(v), t(g), t(beta), s_dev, t(cu, torch.int64), state_out=s_dev)
    np.testing.assert_allclose(n(s_dev), est, rtol=RTOL, atol=ATOL)


def test_null_initial_state_means_zeros():
    q, k, v, g, beta, _ = O.metal_test_inputs(9, 64, 16, 2, 2)
    y, st = gdn_b200.gated_delta_scan_varlen(t(q), t(k), t(v), t(g), t(beta), None)
    ey, est = O.gated_delta_scan(q, k, v, g, beta, np.zeros((2, 16, 64), np.float32))
    np.testing.assert_allclose(n(y), ey, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(n(st)[0], est, rtol=RTOL, atol=ATOL)
