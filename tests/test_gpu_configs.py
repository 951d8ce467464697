"""The BASELINE configurations through the library: config 1 in full
(float32, rel-L2 <= 1e-5), config 3 (T=8192) and config 5 (a stated subset of
its sequences) at full length against the C oracle (bf16 inputs, fp32 state,
rel-L2 <= 2e-3), with the size-independent checks the domain offers."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gpu_helpers import n, t
from oracle import gdn_oracle as O
from oracle import oracle_c

pytestmark = pytest.mark.gpu


def test_config1_float32():
    q, k, v, g_log, beta, s0 = O.config1_inputs(0)
    y, st = gdn_b200.gated_delta_scan(t(q), t(k), t(v), t(g_log), t(beta), t(s0), g_is_log=True)
    ey, est = O.gated_delta_scan(q, k, v, np.exp(g_log.astype(np.float64)), beta, s0)
    assert O.rel_l2(n(y), ey) <= 1e-5
    assert O.rel_l2(n(st), est) <= 1e-5
    # the reference's multiplier convention gives the same result
    y2, st2 = gdn_b200.gated_delta_scan(t(q), t(k), t(v), t(np.exp(g_log)), t(beta), t(s0))
    assert O.rel_l2(n(y2), ey) <= 1e-5


def _bf16_prefill(total, seed, hk=16, hv=32, d=128):
    q, k, v, g_log, beta = O.prefill_inputs(seed, total, hk, hv, d, d)
    return O.bf16_round(q), O.bf16_round(k), O.bf16_round(v), g_log, beta


@pytest.mark.parametrize("algo", ["serial", "auto"])
def test_config3_full_length(algo):
    T = 8192
    q, k, v, g_log, beta = _bf16_prefill(T, 3)
    s0 = np.zeros((1, 32, 128, 128), np.float32)
    y, st = gdn_b200.gated_delta_scan_varlen(
        t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g_log), t(beta), t(s0),
        g_is_log=True, algo=algo,
    )
    ey, est = oracle_c.scan_varlen(q, k, v, g_log, beta, np.array([0, T]), s0, g_is_log=True)
    assert O.rel_l2(n(y), ey) <= 2e-3
    assert O.rel_l2(n(st), est) <= 2e-3


def test_config5_subset_varlen_then_decode():
    lengths = O.config5_lengths()
    sub = lengths[:4]  # sequences 0-3 of the 64 (the full set is 516,496 tokens)
    cu = np.concatenate([[0], np.cumsum(sub)]).astype(np.int64)
    q, k, v, g_log, beta = _bf16_prefill(int(cu[-1]), 5)
    s0 = (np.random.default_rng(2).standard_normal((4, 32, 128, 128)) * 0.02).astype(np.float32)
    state = t(s0)
    y, _ = gdn_b200.gated_delta_scan_varlen(
        t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g_log), t(beta), state,
        t(cu, torch.int64), g_is_log=True, state_out=state,
    )
    ey, est = oracle_c.scan_varlen(q, k, v, g_log, beta, cu, s0, g_is_log=True)
    assert O.rel_l2(n(y), ey) <= 2e-3
    assert O.rel_l2(n(state), est) <= 2e-3
    # then decode steps with the carried states
    for step in range(8):
        dq, dk_, dv_, dg, db, _ = O.decode_inputs(50 + step, 4, 16, 32, 128, 128, with_state=False)
        dq, dk_, dv_ = O.bf16_round(dq), O.bf16_round(dk_), O.bf16_round(dv_)
        yd, _ = gdn_b200.gated_delta_decode(t(dq, torch.bfloat16), t(dk_, torch.bfloat16), t(dv_, torch.bfloat16),
                                            t(dg), t(db), state, g_is_log=True)
        eyd, est = oracle_c.scan_varlen(dq, dk_, dv_, dg, db, np.arange(5), est, g_is_log=True)
        assert O.rel_l2(n(yd), eyd) <= 2e-3
    assert O.rel_l2(n(state), est) <= 2e-3


def test_config2_decode_is_linear_in_v_for_fixed_state():
    """Size-independent property at full config-2 size: with g, beta, q, k and
    the state fixed, y(v1 + v2) - y(v2) = y(v1) - y(0)."""
    B, hk, hv, d = 64, 16, 32, 128
    q, k, v, g_log, beta, s = O.decode_inputs(0, B, hk, hv, d, d)
    qb, kb = t(q, torch.bfloat16), t(k, torch.bfloat16)
    S = t(s)

    def y_of(vv):
        y, _ = gdn_b200.gated_delta_decode(qb, kb, vv, t(g_log), t(beta), S, g_is_log=True, inplace=False)
        return y.double()

    v1 = t(O.bf16_round(v))
    v2 = t(O.bf16_round(np.random.default_rng(1).standard_normal(v.shape).astype(np.float32)))
    zero = torch.zeros_like(v1)
    lhs = y_of(v1 + v2) - y_of(v2)
    rhs = y_of(v1) - y_of(zero)
    assert float((lhs - rhs).norm() / rhs.norm()) < 1e-5
