"""The fused block at one token per sequence (decode through the layer), which
gdn_fused_block runs as a single kernel when Dk = Dv = 128 and the new conv
tail goes to a buffer of its own: against the oracle's restatement of the
layer core (qw/linear_attention.py:81-124) and against the four-kernel chain
(prologue, conv tail, serial scan, epilogue) that the same call takes when
the conv state is updated in place."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200.linear_attention import LinearAttentionShape
from gpu_helpers import dev, n, t
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(B, hk, hv, kernel, seed):
    shape = LinearAttentionShape(hk, hv, 128, 128, kernel)
    rng = np.random.default_rng(seed)
    return shape, dict(
        mixed=O.bf16_round(rng.standard_normal((B, shape.mixed_width)).astype(np.float32)),
        conv_w=(rng.standard_normal((shape.conv_dim, kernel)) * 0.1).astype(np.float32),
        A_log=rng.uniform(0, 1.5, hv).astype(np.float32),
        dt_bias=(rng.standard_normal(hv) * 0.1).astype(np.float32),
        norm_w=(1 + 0.1 * rng.standard_normal(128)).astype(np.float32),
        conv=O.bf16_round(rng.standard_normal((B, kernel - 1, shape.conv_dim)).astype(np.float32)),
        ssm=(rng.standard_normal((B, hv, 128, 128)) * 0.02).astype(np.float32),
    )


def _run(shape, x, act, state_dtype, fused):
    """One token for each sequence; the conv tail to a fresh buffer (the
    single-kernel path) or in place (the chain)."""
    conv = t(x["conv"], state_dtype) if shape.conv_kernel_dim > 1 else None
    ssm = t(x["ssm"])
    conv_out = torch.empty_like(conv) if (fused and conv is not None) else None
    ssm_out = torch.empty_like(ssm)
    out, conv_res, ssm_res = gdn_b200.gated_delta_block(
        t(x["mixed"], act), shape, t(x["conv_w"]), t(x["A_log"]), t(x["dt_bias"]), t(x["norm_w"]), 1e-6, conv, ssm,
        n_seqs=x["mixed"].shape[0], conv_state_out=conv_out, ssm_state_out=ssm_out)
    torch.cuda.synchronize()
    return out, conv_res, ssm_res


def _oracle(shape, x, rnd):
    outs, convs, ssms = [], [], []
    for b in range(x["mixed"].shape[0]):
        o, c, s, _ = O.linear_attention_core(
            x["mixed"][b:b + 1], x["conv_w"], x["conv"][b], x["A_log"], x["dt_bias"], x["norm_w"], x["ssm"][b],
            1e-6, shape.num_key_heads, shape.num_value_heads, 128, 128, rnd=rnd)
        outs.append(o)
        convs.append(c)
        ssms.append(s)
    return np.concatenate(outs), np.stack(convs), np.stack(ssms)


@pytest.mark.parametrize("B,hk,hv,kernel", [(3, 16, 32, 4), (1, 16, 32, 4), (5, 2, 4, 2), (2, 4, 4, 3)])
@pytest.mark.parametrize("state_dtype", [torch.bfloat16, torch.float32])
def test_single_token_block_bf16_matches_oracle_and_chain(B, hk, hv, kernel, state_dtype):
    shape, x = _inputs(B, hk, hv, kernel, seed=B * 10 + kernel)
    eo, ec, es = _oracle(shape, x, O.bf16_round)
    fo, fc, fs = _run(shape, x, torch.bfloat16, state_dtype, fused=True)
    assert O.rel_l2(n(fo), eo) < 2e-3
    assert O.rel_l2(n(fs), es) < 2e-3
    np.testing.assert_array_equal(n(fc), ec)  # the conv tail is a copy of bf16 values
    co, cc, cs = _run(shape, x, torch.bfloat16, state_dtype, fused=False)
    assert O.rel_l2(n(fo), n(co)) < 2e-3
    torch.testing.assert_close(fs, cs, rtol=1e-5, atol=1e-6)
    assert torch.equal(fc, cc)
    gdn_b200.check_device_errors()


def test_single_token_block_float32_matches_oracle():
    shape, x = _inputs(4, 16, 32, 4, seed=77)
    x["mixed"] = np.random.default_rng(78).standard_normal(x["mixed"].shape).astype(np.float32)
    eo, ec, es = _oracle(shape, x, lambda a: a)
    fo, fc, fs = _run(shape, x, torch.float32, torch.float32, fused=True)
    assert O.rel_l2(n(fo), eo) < 1e-5
    assert O.rel_l2(n(fs), es) < 1e-5
    np.testing.assert_allclose(n(fc), ec, rtol=0, atol=0)


def test_single_token_block_without_conv_history_and_in_place_ssm():
    # no conv state (zeros), the ssm state updated in place
    shape, x = _inputs(2, 16, 32, 4, seed=5)
    x["conv"] = np.zeros_like(x["conv"])
    eo, ec, es = _oracle(shape, x, O.bf16_round)
    ssm = t(x["ssm"])
    conv_out = torch.empty(2, 3, shape.conv_dim, device=dev())
    out, _, ssm_res = gdn_b200.gated_delta_block(
        t(x["mixed"], torch.bfloat16), shape, t(x["conv_w"]), t(x["A_log"]), t(x["dt_bias"]), t(x["norm_w"]), 1e-6,
        None, ssm, n_seqs=2, conv_state_out=conv_out)
    assert ssm_res.data_ptr() == ssm.data_ptr()
    assert O.rel_l2(n(out), eo) < 2e-3
    assert O.rel_l2(n(ssm), es) < 2e-3
    np.testing.assert_array_equal(n(conv_out), ec)
