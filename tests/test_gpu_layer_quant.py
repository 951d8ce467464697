"""The linear-attention layer with affine-quantized projections, as the
reference builds it (tests/test_qwen3_5_linear_attention.py:59-91: random
weights quantized to 4 bits with group 64): against the same layer with the
dequantized dense weights (whose parity with the reference's layer the golden
vectors pin), and at the model's head shape in bfloat16 against the oracle's
chain of projection, block and output projection."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200 import LinearWeights, QuantScheme
from gdn_b200.linear_attention import LinearAttentionShape
from gpu_helpers import dev, n, t
from make_golden import LAYER
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

Q = QuantScheme(bits=4, group_size=64)


def _quantized(rng, out_dim, in_dim, scale):
    dense = (rng.standard_normal((out_dim, in_dim)) * scale).astype(np.float32)
    words, s, b = O.quantize_affine(dense, Q.bits, Q.group_size)
    tensors = {"weight": torch.from_numpy(words.view(np.int32)).to(dev()), "scales": t(s, torch.bfloat16),
               "biases": t(b, torch.bfloat16)}
    return tensors, O.dequant_affine(words, s, b, Q.bits, Q.group_size)


def _weights(seed, hidden, shape: LinearAttentionShape, proj_scale):
    rng = np.random.default_rng(seed)
    hv = shape.num_value_heads
    q, d = {}, {}
    for name, rows in (("in_proj_qkv", shape.conv_dim), ("in_proj_z", shape.value_dim), ("in_proj_a", hv),
                       ("in_proj_b", hv)):
        q[name], d[name] = _quantized(rng, rows, hidden, proj_scale)
    q["out_proj"], d["out_proj"] = _quantized(rng, hidden, shape.value_dim, proj_scale)
    other = dict(
        conv1d_weight=(rng.standard_normal((shape.conv_dim, shape.conv_kernel_dim, 1)) * 0.2).astype(np.float32),
        A_log=rng.standard_normal(hv).astype(np.float32),
        dt_bias=rng.standard_normal(hv).astype(np.float32),
        norm_weight=(rng.standard_normal(shape.value_head_dim) * 0.1 + 1.0).astype(np.float32),
    )
    return q, d, other


def _layer(shape, eps, proj, other, quant=None, wrap=lambda x: x):
    return gdn_b200.Qwen3_5LinearAttention(
        shape, eps, wrap(proj["in_proj_qkv"]), wrap(proj["in_proj_z"]), wrap(proj["in_proj_a"]),
        wrap(proj["in_proj_b"]), t(other["conv1d_weight"]), t(other["A_log"]), t(other["dt_bias"]),
        t(other["norm_weight"]), wrap(proj["out_proj"]), quant=quant,
    )


def _cache(shape, dtype=torch.float32):
    return gdn_b200.RecurrentCache(shape.conv_kernel_dim, shape.conv_dim, shape.num_value_heads,
                                   shape.value_head_dim, shape.key_head_dim, device=dev())


SMALL = LinearAttentionShape(LAYER["hk"], LAYER["hv"], LAYER["dk"], LAYER["dv"], LAYER["kernel"])


@pytest.mark.parametrize("wrap_kind", ["dict", "linear_weights"])
def test_quantized_layer_equals_dense_layer_on_dequantized_weights(wrap_kind):
    torch.backends.cuda.matmul.allow_tf32 = False
    q, d, other = _weights(0, LAYER["hidden"], SMALL, 0.05)
    dense = _layer(SMALL, LAYER["eps"], {k: t(v) for k, v in d.items()}, other)
    if wrap_kind == "dict":
        quant = _layer(SMALL, LAYER["eps"], q, other, quant=Q)
    else:
        quant = _layer(SMALL, LAYER["eps"], q, other, wrap=lambda w: LinearWeights(w, Q))
    rng = np.random.default_rng(7)
    c_dense, c_quant = _cache(SMALL), _cache(SMALL)
    for L in (6, 1, 1, 3):  # prefill, two decode steps, a chunk: the cache carries through
        x = t(rng.standard_normal((L, LAYER["hidden"])).astype(np.float32))
        a = dense(x if L > 1 else x[0], c_dense)
        b = quant(x if L > 1 else x[0], c_quant)
        torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(c_quant.ssm_state, c_dense.ssm_state, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(c_quant.conv_state, c_dense.conv_state, rtol=1e-5, atol=1e-6)
    assert c_quant.size == 11


def test_mixed_storage_projections():
    # a dense in_proj_a beside quantized others: computed per projection
    torch.backends.cuda.matmul.allow_tf32 = False
    q, d, other = _weights(1, LAYER["hidden"], SMALL, 0.05)
    mixed = dict(q)
    mixed["in_proj_a"] = t(d["in_proj_a"])
    dense = _layer(SMALL, LAYER["eps"], {k: t(v) for k, v in d.items()}, other)
    layer = _layer(SMALL, LAYER["eps"], mixed, other, quant=Q)
    assert layer.in_proj is None
    x = t(np.random.default_rng(3).standard_normal((5, LAYER["hidden"])).astype(np.float32))
    torch.testing.assert_close(layer(x, _cache(SMALL)), dense(x, _cache(SMALL)), rtol=1e-5, atol=1e-6)


def test_quantized_layer_bf16_at_model_shape():
    shape = LinearAttentionShape(16, 32, 128, 128, 4)
    hidden, eps = 2048, 1e-6
    q, d, other = _weights(2, hidden, shape, 0.02)
    layer = _layer(shape, eps, q, other, quant=Q)
    rng = np.random.default_rng(5)
    cache = _cache(shape)
    conv = np.zeros((3, shape.conv_dim), np.float32)
    ssm = np.zeros((32, 128, 128), np.float32)
    for L in (150, 1, 40):
        x = O.bf16_round(rng.standard_normal((L, hidden)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        mixed = O.bf16_round((x.astype(np.float64) @ d_in(d).T).astype(np.float32))
        core, conv, ssm, _ = O.linear_attention_core(
            mixed, other["conv1d_weight"].reshape(shape.conv_dim, 4), conv, other["A_log"], other["dt_bias"],
            other["norm_weight"], ssm, eps, 16, 32, 128, 128, rnd=O.bf16_round)
        conv = O.bf16_round(conv)
        want = core.reshape(L, -1).astype(np.float64) @ d["out_proj"].astype(np.float64).T
        assert O.rel_l2(n(got), want) < 5e-3
    assert O.rel_l2(n(cache.ssm_state), ssm) < 5e-3
    assert cache.size == 191


def d_in(d):
    # the mixed row's projection order: q|k|v (in_proj_qkv), z, b, a
    return np.concatenate([d["in_proj_qkv"], d["in_proj_z"], d["in_proj_b"], d["in_proj_a"]]).astype(np.float64)
