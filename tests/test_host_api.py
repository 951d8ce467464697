"""Host-side behaviour of the Python API that needs no GPU: the reference's
shape checks and messages (qw/gated_delta.py:57-79, tested by the reference
at tests/test_gated_delta_metal.py:137-156), refusal of CPU tensors (there is
no CPU path), and the RecurrentCache contract."""

from __future__ import annotations

import pytest
import torch

import gdn_b200
from gdn_b200.linear_attention import LinearAttentionShape
from oracle import gdn_oracle as O


def _inputs():
    return [torch.from_numpy(a) for a in O.metal_test_inputs(5)]


@pytest.mark.parametrize("invalid", ["k", "v", "g", "beta", "state", "heads", "empty"])
def test_invalid_shapes_are_rejected_before_dispatch(invalid):
    inputs = _inputs()
    index = {"k": 1, "v": 2, "g": 3, "beta": 4, "state": 5}
    if invalid in index:
        inputs[index[invalid]] = inputs[index[invalid]][:1]
    elif invalid == "heads":
        inputs[0] = inputs[0][:, :1].repeat(1, 3, 1)
        inputs[1] = inputs[0]
    else:
        inputs = [a[:0] for a in inputs[:-1]] + inputs[-1:]
    with pytest.raises(ValueError) as err:
        gdn_b200.gated_delta_scan(*inputs)
    assert "CUDA" not in str(err.value)  # a shape error, found before anything else


def test_cpu_tensors_are_refused_not_computed():
    with pytest.raises(ValueError, match="CUDA tensors only"):
        gdn_b200.gated_delta_scan(*_inputs())


def test_recurrent_cache_layout_and_update():
    with pytest.raises(ValueError, match="conv_kernel_dim must be positive"):
        gdn_b200.RecurrentCache(0, 8, 2, 4, 4, device="cpu")
    cache = gdn_b200.RecurrentCache(4, 256, 4, 32, 16, dtype=torch.bfloat16, device="cpu")
    conv, ssm = cache.state()
    assert conv.shape == (3, 256) and conv.dtype == torch.bfloat16
    assert ssm.shape == (4, 32, 16) and ssm.dtype == torch.float32  # float32 whatever the dtype
    cache.update(conv + 1, ssm + 1, advance=5)
    cache.update(*cache.state(), advance=2)
    assert cache.size == 7
    b = gdn_b200.BatchedRecurrentCache(3, 4, 256, 4, 32, 16, device="cpu")
    assert b.state()[1].shape == (3, 4, 32, 16)
    b.advance([1, 2, 3])
    assert b.sizes == [1, 2, 3]


def test_linear_attention_shape():
    s = LinearAttentionShape(16, 32, 128, 128, 4)
    assert s.conv_dim == 8192 and s.mixed_width == 12352


def test_decode_plan_rejects_cpu_tensors():
    import gdn_b200

    x = torch.zeros(2, 1, 8)
    with pytest.raises(ValueError, match="CUDA"):
        gdn_b200.DecodePlan(x, x, x, torch.zeros(2, 1), torch.zeros(2, 1), torch.zeros(2, 1, 8, 8))


def test_attention_layer_fuses_projections_sharing_a_storage_scheme():
    from gdn_b200 import AttentionShape, QuantScheme, Qwen3_5Attention

    shape = AttentionShape(4, 2, 32, 16, 10000.0)
    dense = lambda o, i: torch.randn(o, i)
    layer = Qwen3_5Attention(shape, 1e-6, dense(256, 64), torch.ones(32), dense(64, 64), torch.ones(32),
                             dense(64, 64), dense(64, 128))
    assert layer.qkv_proj is not None and layer.qkv_proj.tensors.shape == (384, 64)
    torch.testing.assert_close(layer.qkv_proj.tensors[256:320], layer.k_proj.tensors)
    q4 = QuantScheme(bits=4, group_size=64)
    quantized_k = {"weight": torch.zeros(64, 8, dtype=torch.int32), "scales": torch.ones(64, 1).bfloat16()}
    mixed = Qwen3_5Attention(shape, 1e-6, dense(256, 64), torch.ones(32), gdn_b200.LinearWeights(quantized_k, q4),
                             torch.ones(32), dense(64, 64), dense(64, 128))
    assert mixed.qkv_proj is None  # one projection stored differently: three products
