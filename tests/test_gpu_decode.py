"""The HBM-bound decode step (gdn_decode) against the oracle: config 2's
shapes (bf16 q/k/v, fp32 state), several Dk, state slots, in place and out
of place, and 100 carried steps. The decode computes in float32 on the same
bf16 inputs as the oracle, so it is held to rel-L2 1e-5 (the north-star
bound for bf16 inputs is 2e-3)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gpu_helpers import n, t
from oracle import gdn_oracle as O
from oracle import oracle_c

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _bf(x):
    return O.bf16_round(x)


@pytest.mark.parametrize("dk,dv,hk,hv", [(128, 128, 16, 32), (64, 64, 4, 8), (256, 7, 2, 6), (32, 5, 3, 6),
                                         (16, 8, 2, 6), (128, 17, 2, 4)])
def test_decode_step_matches_oracle(dk, dv, hk, hv):
    B = 8
    q, k, v, g_log, beta, s = O.decode_inputs(3, B, hk, hv, dk, dv)
    q, k, v = _bf(q), _bf(k), _bf(v)
    y, st = gdn_b200.gated_delta_decode(t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16),
                                        t(g_log), t(beta), t(s), g_is_log=True, inplace=False)
    ey, est = oracle_c.scan_varlen(q, k, v, g_log, beta, np.arange(B + 1), s, g_is_log=True)
    assert O.rel_l2(n(y), ey) < TOL
    assert O.rel_l2(n(st), est) < TOL


def test_config2_full_batch_100_carried_steps_in_place():
    B, hk, hv, d = 64, 16, 32, 128
    _, _, _, _, _, s = O.decode_inputs(0, B, hk, hv, d, d)
    state = t(s)
    ref_state = s[:4].copy()  # oracle on the first 4 sequences, all 100 steps
    for step in range(100):
        q, k, v, g_log, beta, _ = O.decode_inputs(1000 + step, B, hk, hv, d, d, with_state=False)
        q, k, v = _bf(q), _bf(k), _bf(v)
        y, _ = gdn_b200.gated_delta_decode(t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16),
                                           t(g_log), t(beta), state, g_is_log=True)
        ey, ref_state = oracle_c.scan_varlen(q[:4], k[:4], v[:4], g_log[:4], beta[:4], np.arange(5), ref_state,
                                             g_is_log=True)
        if step in (0, 99):
            assert O.rel_l2(n(y)[:4], ey) < TOL
    assert O.rel_l2(n(state)[:4], ref_state) < TOL
    assert torch.isfinite(state).all()


def test_decode_state_slots_update_only_their_rows():
    B, slots, hk, hv, d = 4, 10, 2, 4, 64
    q, k, v, g_log, beta, _ = O.decode_inputs(5, B, hk, hv, d, d, with_state=False)
    pool = (np.random.default_rng(6).standard_normal((slots, hv, d, d)) * 0.02).astype(np.float32)
    idx = np.array([7, 2, 9, 0], np.int32)
    pool_dev = t(pool)
    y, _ = gdn_b200.gated_delta_decode(t(q), t(k), t(v), t(g_log), t(beta), pool_dev, g_is_log=True,
                                       state_slots=t(idx, torch.int32))
    ey, est = oracle_c.scan_varlen(q, k, v, g_log, beta, np.arange(B + 1), pool[idx], g_is_log=True)
    got = n(pool_dev)
    assert O.rel_l2(n(y), ey) < TOL
    assert O.rel_l2(got[idx], est) < TOL
    untouched = [i for i in range(slots) if i not in idx]
    np.testing.assert_array_equal(got[untouched], pool[untouched])


def test_decode_multiplier_gate_and_bf16_output():
    q, k, v, g_log, beta, s = O.decode_inputs(9, 4, 2, 4, 128, 128)
    g = np.exp(g_log)
    y, st = gdn_b200.gated_delta_decode(t(q), t(k), t(v), t(g), t(beta), t(s), inplace=False,
                                        out_dtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    ey, est = oracle_c.scan_varlen(q, k, v, g, beta, np.arange(5), s)
    assert O.rel_l2(n(y), ey) < 4e-3  # bf16 rounding of the output
    assert O.rel_l2(n(st), est) < TOL


def test_decode_plan_matches_the_call_over_steps_and_slots():
    # a fixed-buffer decode loop: new contents every step, one prepared call
    bsz, hk, hv, d = 6, 2, 4, 64
    q0, k0, v0, g0, b0, s0 = O.decode_inputs(21, bsz, hk, hv, d, d)
    q, k, v = (t(x, torch.bfloat16) for x in (q0, k0, v0))
    g, beta = t(g0), t(b0)
    pool = t(np.concatenate([s0, s0 * 0.5]))  # 12 slots, this batch uses 6 of them
    slots = torch.tensor([7, 0, 3, 11, 5, 9], dtype=torch.int32, device=q.device)
    ref_pool = pool.clone()
    plan = gdn_b200.DecodePlan(q, k, v, g, beta, pool, g_is_log=True, state_slots=slots)
    for step in range(4):
        qs, ks, vs, gs, bs, _ = O.decode_inputs(100 + step, bsz, hk, hv, d, d)
        for dst, src in ((q, qs), (k, ks), (v, vs), (g, gs), (beta, bs)):
            dst.copy_(t(src, dst.dtype))
        y_ref, _ = gdn_b200.gated_delta_decode(q, k, v, g, beta, ref_pool, g_is_log=True, state_slots=slots)
        y = plan.run()
        torch.testing.assert_close(y, y_ref, rtol=0, atol=0)
    torch.testing.assert_close(pool, ref_pool, rtol=0, atol=0)
    with pytest.raises(ValueError, match="never copies|one supported dtype"):
        gdn_b200.DecodePlan(q.double(), k.double(), v.double(), g, beta, pool, state_slots=slots)
    with pytest.raises(ValueError, match="g and beta"):
        gdn_b200.DecodePlan(q, k, v, g.double(), beta, pool, state_slots=slots)
