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


# ---------------------------------------------------------------------------
# Config 4 at its stated size: the fused block over B=8 sequences of T=4096
# tokens at the model's head shape (16 key / 32 value heads of 128, hidden
# 2048), bf16 mixed projection ~ N(0,1), conv_w ~ N(0,0.1), A_log ~ U(0,1.5),
# dt_bias ~ N(0,0.1), zero conv state and zero S0; norm_w = 1 and N(1,0.1).
# Oracle: the reference layer's steps (qw/linear_attention.py:96-124) with
# bf16 rounding where the reference materialises bf16 arrays, the scan in
# float64 by the C oracle over all 8 sequences.
# ---------------------------------------------------------------------------
C4_B, C4_T, C4_HK, C4_HV, C4_D = 8, 4096, 16, 32, 128


@pytest.fixture(scope="module")
def config4_case():
    mixed, conv_w, A_log, dt_bias, _ = O.block_inputs(4, C4_B, C4_T, C4_HK, C4_HV, C4_D, C4_D)
    mixed = O.bf16_round(mixed)
    conv0 = np.zeros((3, 2 * C4_HK * C4_D + C4_HV * C4_D), np.float32)
    parts = [O.block_prologue(mixed[b * C4_T:(b + 1) * C4_T], conv_w, conv0, A_log, dt_bias,
                              C4_HK, C4_HV, C4_D, C4_D, rnd=O.bf16_round) for b in range(C4_B)]
    q, k, v, g_log, beta = (np.concatenate([p[i] for p in parts]) for i in range(5))
    cu = np.arange(C4_B + 1, dtype=np.int64) * C4_T
    s0 = np.zeros((C4_B, C4_HV, C4_D, C4_D), np.float32)
    y, s_end = oracle_c.scan_varlen(q, k, v, g_log, beta, cu, s0, g_is_log=True)
    _, z, _, _ = O.split_mixed(mixed, C4_HK, C4_HV, C4_D, C4_D)
    return {"mixed": mixed, "conv_w": conv_w, "A_log": A_log, "dt_bias": dt_bias, "y": y, "state": s_end,
            "z": z.reshape(-1, C4_HV, C4_D), "conv_tail": np.stack([p[5] for p in parts])}


@pytest.mark.parametrize("norm", ["ones", "n1_0.1"])
def test_config4_full_size_fused_block(config4_case, norm):
    from gdn_b200.linear_attention import LinearAttentionShape

    c = config4_case
    norm_w = np.ones(C4_D, np.float32) if norm == "ones" else \
        (1 + 0.1 * np.random.default_rng(44).standard_normal(C4_D)).astype(np.float32)
    shape = LinearAttentionShape(C4_HK, C4_HV, C4_D, C4_D, 4)
    conv_state = torch.zeros(C4_B, 3, shape.conv_dim, device="cuda")
    ssm = torch.zeros(C4_B, C4_HV, C4_D, C4_D, device="cuda")
    out, _, _ = gdn_b200.gated_delta_block(t(c["mixed"], torch.bfloat16), shape, t(c["conv_w"]), t(c["A_log"]),
                                           t(c["dt_bias"]), t(norm_w), 1e-6, conv_state, ssm, n_seqs=C4_B)
    gdn_b200.check_device_errors()
    expected = O.gated_rms_norm(O.bf16_round(c["y"]), c["z"], norm_w, 1e-6, rnd=O.bf16_round)
    got = n(out)
    assert np.isfinite(got).all()
    assert O.rel_l2(got, expected) <= 2e-3, O.rel_l2(got, expected)
    assert O.rel_l2(n(ssm), c["state"]) <= 2e-3, O.rel_l2(n(ssm), c["state"])
    np.testing.assert_array_equal(n(conv_state), c["conv_tail"])


def test_config5_shortest_and_longest_through_the_lpt_partition():
    """Config 5's 8 shortest sequences and its longest, split over two ranks
    by the bench's LPT partition and run rank by rank (one packed prefill per
    rank's share), then decode steps with the carried states."""
    from gdn_b200.sharding import lpt_partition

    lengths = O.config5_lengths()
    order = np.argsort(lengths, kind="stable")
    chosen = [int(i) for i in order[:8]] + [int(order[-1])]
    sub = lengths[chosen]
    assert sub.max() == lengths.max() and len(sub) == 9
    for share in lpt_partition(sub, 2):
        ln = sub[share]
        cu = np.concatenate([[0], np.cumsum(ln)]).astype(np.int64)
        q, k, v, g_log, beta = _bf16_prefill(int(cu[-1]), 50 + len(share))
        s0 = (np.random.default_rng(len(share)).standard_normal((len(ln), 32, 128, 128)) * 0.02).astype(np.float32)
        state = t(s0)
        y, _ = gdn_b200.gated_delta_scan_varlen(
            t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g_log), t(beta), state,
            t(cu, torch.int64), g_is_log=True, state_out=state,
        )
        ey, est = oracle_c.scan_varlen(q, k, v, g_log, beta, cu, s0, g_is_log=True)
        assert O.rel_l2(n(y), ey) <= 2e-3
        assert O.rel_l2(n(state), est) <= 2e-3
        for step in range(4):
            dq, dk_, dv_, dg, db, _ = O.decode_inputs(80 + step, len(ln), 16, 32, 128, 128, with_state=False)
            dq, dk_, dv_ = O.bf16_round(dq), O.bf16_round(dk_), O.bf16_round(dv_)
            yd, _ = gdn_b200.gated_delta_decode(t(dq, torch.bfloat16), t(dk_, torch.bfloat16),
                                                t(dv_, torch.bfloat16), t(dg), t(db), state, g_is_log=True)
            eyd, est = oracle_c.scan_varlen(dq, dk_, dv_, dg, db, np.arange(len(ln) + 1), est, g_is_log=True)
            assert O.rel_l2(n(yd), eyd) <= 2e-3
        assert O.rel_l2(n(state), est) <= 2e-3
