"""The chunked tensor-core prefill (gdn_scan with algo=chunked: chunk 64,
Dk = Dv = 128, bf16 q/k/v, fp32 state) against the C oracle's float64
recurrence on the same bf16 inputs.

Bound: the north star's rel-L2 <= 2e-3 for bf16 inputs. The design (tf32
tensor-core operands: the float32 state read as tf32 from tensor memory, the
other tf32 operands rounded to nearest, the state update's Delta' as bf16
hi + lo against exact bf16 K) gives ~3e-4 to 5e-4 in a float64 emulation at
T = 2048 for the decays below; it is held to 1e-3 here, half the bound, so
that a precision regression shows before the bound is reached."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gpu_helpers import n, t
from oracle import gdn_oracle as O
from oracle import oracle_c

pytestmark = pytest.mark.gpu
BOUND = 2e-3
DESIGN = 1e-3


def _inputs(lengths, hk, hv, seed, decay="cfg", state_std=0.02):
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    N = int(cu[-1])
    q, k, v, g_log, beta = O.prefill_inputs(seed, N, hk, hv, 128, 128)
    q, k, v = O.bf16_round(q), O.bf16_round(k), O.bf16_round(v)
    rng = np.random.default_rng(seed + 1)
    if decay == "slow":  # reference test distribution: g ~ U(0.98, 1)
        g_log = np.log(rng.uniform(0.98, 1, g_log.shape)).astype(np.float32)
    elif decay == "strong":  # config 4: -exp(A_log) softplus(a + dt_bias), A_log ~ U(0, 1.5)
        A_log = rng.uniform(0, 1.5, hv).astype(np.float32)
        g_log = O.forget_gate_log(rng.standard_normal(g_log.shape).astype(np.float32), A_log,
                                  (rng.standard_normal(hv) * 0.1).astype(np.float32))
    s0 = (rng.standard_normal((len(lengths), hv, 128, 128)) * state_std).astype(np.float32)
    return q, k, v, g_log, beta, cu, s0


def _run(q, k, v, g, beta, cu, s0, algo="chunked", g_is_log=True, out_dtype=torch.float32, inplace=False):
    state = t(s0)
    y, st = gdn_b200.gated_delta_scan_varlen(
        t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g), t(beta), state,
        t(cu, torch.int64), g_is_log=g_is_log, algo=algo, out_dtype=out_dtype,
        state_out=state if inplace else None,
    )
    gdn_b200.check_device_errors()
    return n(y), n(st)


@pytest.mark.parametrize("decay", ["cfg", "slow", "strong"])
def test_chunked_single_sequence_matches_oracle(decay):
    q, k, v, g, beta, cu, s0 = _inputs([1000], 4, 8, seed=1, decay=decay)
    y, st = _run(q, k, v, g, beta, cu, s0)
    ey, est = oracle_c.scan_varlen(q, k, v, g, beta, cu, s0, g_is_log=True)
    assert O.rel_l2(y, ey) <= DESIGN, O.rel_l2(y, ey)
    assert O.rel_l2(st, est) <= DESIGN, O.rel_l2(st, est)


def test_chunked_varlen_edges_in_place():
    lengths = [1, 63, 64, 65, 0, 200, 128, 7]
    q, k, v, g, beta, cu, s0 = _inputs(lengths, 2, 4, seed=2)
    y, st = _run(q, k, v, g, beta, cu, s0, inplace=True)
    ey, est = oracle_c.scan_varlen(q, k, v, g, beta, cu, s0, g_is_log=True)
    assert O.rel_l2(y, ey) <= DESIGN
    assert O.rel_l2(st, est) <= DESIGN
    np.testing.assert_array_equal(st[4], s0[4])  # the empty sequence keeps its state
    for b in range(len(lengths)):  # every sequence, not just the aggregate
        s, e = cu[b], cu[b + 1]
        if e > s:
            assert O.rel_l2(y[s:e], ey[s:e]) <= DESIGN
        assert O.rel_l2(st[b], est[b]) <= DESIGN


def test_chunked_multiplier_gates_bf16_output_and_zero_state():
    q, k, v, g, beta, cu, s0 = _inputs([300, 129], 2, 4, seed=3)
    s0[:] = 0
    y, st = _run(q, k, v, np.exp(g), beta, cu, s0, g_is_log=False, out_dtype=torch.bfloat16)
    ey, est = oracle_c.scan_varlen(q, k, v, np.exp(g), beta, cu, s0)
    assert O.rel_l2(y, ey) <= 4e-3  # bf16 rounding of the output itself
    assert O.rel_l2(st, est) <= DESIGN


def test_chunked_and_serial_agree():
    q, k, v, g, beta, cu, s0 = _inputs([777], 16, 32, seed=4)
    yc, sc = _run(q, k, v, g, beta, cu, s0, algo="chunked")
    ys, ss = _run(q, k, v, g, beta, cu, s0, algo="serial")
    assert O.rel_l2(yc, ys) <= DESIGN
    assert O.rel_l2(sc, ss) <= DESIGN


def test_reference_known_answer_shape_through_chunked_path(golden):
    # tests/test_gated_delta_metal.py's (17, 128, 128, 16, 32) case, q/k/v rounded to bf16
    q, k, v, g, beta, s0 = O.metal_test_inputs(300, 128, 128, 16, 32)
    q, k, v = O.bf16_round(q), O.bf16_round(k), O.bf16_round(v)
    cu = np.array([0, 300])
    y, st = _run(q, k, v, g, beta, cu, s0[None], g_is_log=False)
    ey, est = O.gated_delta_scan(q, k, v, g, beta, s0)
    assert O.rel_l2(y, ey) <= DESIGN
    assert O.rel_l2(st[0], est) <= DESIGN


def test_chunked_rejects_unsupported_shapes():
    q, k, v, g, beta, cu, s0 = _inputs([100], 2, 4, seed=5)
    with pytest.raises(ValueError, match="chunked"):
        gdn_b200.gated_delta_scan_varlen(t(q[:, :, :64]), t(k[:, :, :64]), t(v), t(g), t(beta), None,
                                         algo="chunked", g_is_log=True)


@pytest.mark.parametrize("hk,hv,T,decay", [(4, 8, 4096, "cfg"), (8, 16, 3072 + 40, "slow"),
                                           (16, 32, 2048, "strong"), (16, 32, 1600, "cfg")])
def test_segmented_single_sequence(hk, hv, T, decay):
    """One dense sequence (no cu_seqlens) whose heads leave the GPU idle is run
    in time segments (transition chains + start-state combine); it must agree
    with the oracle's serial recurrence and with the unsegmented chunked run."""
    q, k, v, g, beta, cu, s0 = _inputs([T], hk, hv, seed=7, decay=decay, state_std=0.05)
    state = t(s0)
    y, st = gdn_b200.gated_delta_scan_varlen(
        t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g), t(beta), state,
        g_is_log=True, algo="chunked", state_out=state)  # in place
    gdn_b200.check_device_errors()
    y, st = n(y), n(st)
    ey, est = oracle_c.scan_varlen(q, k, v, g, beta, cu, s0, g_is_log=True)
    assert O.rel_l2(y, ey) <= DESIGN, O.rel_l2(y, ey)
    assert O.rel_l2(st, est) <= DESIGN, O.rel_l2(st, est)
    y1, st1 = _run(q, k, v, g, beta, cu, s0)  # with cu_seqlens: one chain per head
    assert O.rel_l2(y, y1) <= DESIGN and O.rel_l2(st, st1) <= DESIGN
