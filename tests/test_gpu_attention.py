"""The softmax-attention layer (gdn_attention) against the reference's own
Qwen3_5Attention + GrowingKVCache (golden vectors, float32) and against the
oracle's restatement with bf16 rounding at the model's head shape."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200 import AttentionShape, GrowingKVCache, Qwen3_5Attention
from gpu_helpers import dev, n, t
from make_golden import ATTN, attn_case
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

SMALL = AttentionShape(ATTN["heads"], ATTN["kv_heads"], ATTN["head_dim"], ATTN["rotary"], ATTN["theta"])


def _layer(w, shape=SMALL, eps=ATTN["eps"], dtype=torch.float32):
    return Qwen3_5Attention(shape, eps, t(w["q_proj"], dtype), t(w["q_norm"]), t(w["k_proj"], dtype),
                            t(w["k_norm"]), t(w["v_proj"], dtype), t(w["o_proj"], dtype))


def _cache(shape=SMALL, max_context=16, dtype=torch.float32):
    return GrowingKVCache(max_context, shape.num_key_value_heads, shape.head_dim, dtype=dtype, device=dev())


@pytest.mark.parametrize("seq_len", [1, 6])
def test_attention_matches_reference_layer(seq_len, golden):
    torch.backends.cuda.matmul.allow_tf32 = False
    w = attn_case(0)
    x = np.random.default_rng(200).standard_normal((seq_len, ATTN["hidden"])).astype(np.float32)
    cache = _cache()
    out = _layer(w)(t(x), cache)
    np.testing.assert_allclose(n(out), golden[f"attn_fresh_{seq_len}/out"], rtol=1e-4, atol=1e-5)
    keys, values = cache.state()
    np.testing.assert_allclose(n(keys), golden[f"attn_fresh_{seq_len}/keys"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n(values), golden[f"attn_fresh_{seq_len}/values"], rtol=1e-5, atol=1e-6)
    assert cache.size == seq_len


def test_attention_decode_steps_and_offset_chunks(golden):
    torch.backends.cuda.matmul.allow_tf32 = False
    w = attn_case(1)
    x = np.random.default_rng(201).standard_normal((5, ATTN["hidden"])).astype(np.float32)
    layer, cache = _layer(w), _cache()
    stepwise = torch.stack([layer(t(x[i]), cache) for i in range(5)])
    np.testing.assert_allclose(n(stepwise), golden["attn_steps/out"], rtol=1e-4, atol=1e-5)
    batched = layer(t(x), _cache())
    np.testing.assert_allclose(n(batched), golden["attn_steps/batched"], rtol=1e-4, atol=1e-5)

    w = attn_case(3)
    xs = np.random.default_rng(203).standard_normal((3, 4, ATTN["hidden"])).astype(np.float32)
    layer, cache = _layer(w), _cache()
    outs = torch.cat([layer(t(xc), cache) for xc in xs])
    np.testing.assert_allclose(n(outs), golden["attn_chunks/out"], rtol=1e-4, atol=1e-5)
    keys, values = cache.state()
    np.testing.assert_allclose(n(keys), golden["attn_chunks/keys"], rtol=1e-5, atol=1e-6)
    assert cache.size == 12


def _random_weights(rng, shape, hidden, scale):
    h, hkv, hd = shape.num_attention_heads, shape.num_key_value_heads, shape.head_dim
    dense = lambda o, i: (rng.standard_normal((o, i)) * scale).astype(np.float32)
    w = {"q_proj": dense(h * hd * 2, hidden), "k_proj": dense(hkv * hd, hidden), "v_proj": dense(hkv * hd, hidden),
         "o_proj": dense(hidden, h * hd)}
    w["q_norm"] = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    w["k_norm"] = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    return w


def _bf16_weights(w):
    return {k: (O.bf16_round(v) if k.endswith("proj") else v) for k, v in w.items()}


def test_attention_bf16_at_model_shape_prefill_growth_and_decode():
    # the model's attention heads: 16 queries over 2 key/value heads of 256, rotary 64
    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    hidden, eps = 2048, 1e-6
    rng = np.random.default_rng(11)
    w = _bf16_weights(_random_weights(rng, shape, hidden, 0.02))
    layer = _layer(w, shape, eps, torch.bfloat16)
    cache = _cache(shape, max_context=1024, dtype=torch.bfloat16)
    keys = np.zeros((2, 0, 256))
    values = np.zeros((2, 0, 256))
    for L in (250, 10, 1, 1, 3):  # crosses the 256-token growth block; decode rows take the key splits
        x = O.bf16_round(rng.standard_normal((L, hidden)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        want, keys, values = O.attention_layer(x, w, keys, values, 16, 2, 256, 64, 10000000.0, eps,
                                               rnd=O.bf16_round)
        assert O.rel_l2(n(got), want) < 1e-2, (L, O.rel_l2(n(got), want))
    assert cache.size == 265 and cache.allocated_size == 512
    gk, gv = cache.state()
    assert O.rel_l2(n(gk), keys) < 1e-2 and O.rel_l2(n(gv), values) < 1e-2


@pytest.mark.parametrize("heads,kv_heads,head_dim,rotary", [(8, 8, 64, 64), (6, 2, 128, 32), (4, 1, 256, 0)])
def test_attention_float32_other_head_shapes(heads, kv_heads, head_dim, rotary):
    torch.backends.cuda.matmul.allow_tf32 = False
    shape = AttentionShape(heads, kv_heads, head_dim, rotary, 10000.0)
    rng = np.random.default_rng(heads + head_dim)
    w = _random_weights(rng, shape, 96, 0.1)
    layer, cache = _layer(w, shape, 1e-6), _cache(shape, max_context=300)
    keys, values = np.zeros((kv_heads, 0, head_dim)), np.zeros((kv_heads, 0, head_dim))
    for L in (37, 1, 140):
        x = rng.standard_normal((L, 96)).astype(np.float32)
        got = layer(t(x), cache)
        want, keys, values = O.attention_layer(x, w, keys, values, heads, kv_heads, head_dim, rotary, 10000.0, 1e-6)
        np.testing.assert_allclose(n(got), want, rtol=2e-4, atol=2e-5)


def test_cache_capacity_is_a_hard_limit():
    cache = _cache(max_context=4)
    w = attn_case(0)
    layer = _layer(w)
    layer(t(np.zeros((3, ATTN["hidden"]), np.float32)), cache)
    with pytest.raises(IndexError):
        layer(t(np.zeros((2, ATTN["hidden"]), np.float32)), cache)
    assert cache.size == 3
    gdn_b200.check_device_errors()


@pytest.mark.parametrize("heads,kv_heads,head_dim,rotary", [(8, 2, 64, 16), (4, 4, 128, 128), (16, 4, 256, 64)])
def test_attention_bf16_tensor_core_prefill(heads, kv_heads, head_dim, rotary):
    # enough rows for one key split: the mma.sync prefill, then a second
    # chunk whose queries start at an offset (the causal mask off the diagonal)
    shape = AttentionShape(heads, kv_heads, head_dim, rotary, 1000000.0)
    hidden = 256
    rng = np.random.default_rng(head_dim + heads)
    w = _bf16_weights(_random_weights(rng, shape, hidden, 0.05))
    layer = _layer(w, shape, 1e-6, torch.bfloat16)
    cache = _cache(shape, max_context=1024, dtype=torch.bfloat16)
    keys, values = np.zeros((kv_heads, 0, head_dim)), np.zeros((kv_heads, 0, head_dim))
    for L in (130, 300):
        x = O.bf16_round(rng.standard_normal((L, hidden)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        want, keys, values = O.attention_layer(x, w, keys, values, heads, kv_heads, head_dim, rotary, 1000000.0,
                                               1e-6, rnd=O.bf16_round)
        assert O.rel_l2(n(got), want) < 1e-2, (L, O.rel_l2(n(got), want))


def _quantized(w):
    """The reference test's construction (tests/test_qwen3_5_attention.py:64-71):
    4-bit, group 64 projections and the dequantized dense copy."""
    from gdn_b200 import QuantScheme

    q, d = {}, {}
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        words, s, b = O.quantize_affine(w[name], 4, 64)
        q[name] = {"weight": torch.from_numpy(words.view(np.int32)).to(dev()), "scales": t(s, torch.bfloat16),
                   "biases": t(b, torch.bfloat16)}
        d[name] = O.dequant_affine(words, s, b, 4, 64)
    return q, d, QuantScheme(bits=4, group_size=64)


def test_quantized_attention_equals_dense_on_dequantized_weights():
    torch.backends.cuda.matmul.allow_tf32 = False
    w = attn_case(0)
    q, d, quant = _quantized(w)
    qlayer = Qwen3_5Attention(SMALL, ATTN["eps"], q["q_proj"], t(w["q_norm"]), q["k_proj"], t(w["k_norm"]),
                              q["v_proj"], q["o_proj"], quant=quant)
    dlayer = _layer({**w, **d})
    cq, cd = _cache(), _cache()
    rng = np.random.default_rng(5)
    for L in (6, 1, 3):
        x = t(rng.standard_normal((L, ATTN["hidden"])).astype(np.float32))
        torch.testing.assert_close(qlayer(x if L > 1 else x[0], cq), dlayer(x if L > 1 else x[0], cd),
                                   rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(cq.state()[0], cd.state()[0], rtol=1e-5, atol=1e-6)


def test_quantized_attention_bf16_model_shape():
    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    rng = np.random.default_rng(17)
    w = _random_weights(rng, shape, 2048, 0.02)
    q, d, quant = _quantized(w)
    layer = Qwen3_5Attention(shape, 1e-6, q["q_proj"], t(w["q_norm"]), q["k_proj"], t(w["k_norm"]), q["v_proj"],
                             q["o_proj"], quant=quant)
    cache = _cache(shape, max_context=512, dtype=torch.bfloat16)
    keys, values = np.zeros((2, 0, 256)), np.zeros((2, 0, 256))
    dw = {**w, **d}
    for L in (200, 1):  # the GEMM and tensor-core prefill, then the GEMV and split-key decode
        x = O.bf16_round(rng.standard_normal((L, 2048)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        want, keys, values = O.attention_layer(x, dw, keys, values, 16, 2, 256, 64, 10000000.0, 1e-6,
                                               rnd=O.bf16_round)
        assert O.rel_l2(n(got), want) < 1e-2, (L, O.rel_l2(n(got), want))


def test_decode_captured_in_a_cuda_graph_equals_the_eager_call():
    # the attention and combine kernels are launched as programmatic
    # dependents of the kernel before them; a captured replay must give the
    # eager call's bits
    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    rng = np.random.default_rng(23)
    L = 300
    bf = lambda *s: t(O.bf16_round(rng.standard_normal(s).astype(np.float32)), torch.bfloat16)
    qg, k, v = bf(L, 16 * 512), bf(L, 512), bf(L, 512)
    qn = t((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    kn = t((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))

    def filled():
        cache = GrowingKVCache(L + 8, 2, 256, dtype=torch.bfloat16, device=dev())
        gdn_b200.attention_core(qg[:L - 1], k[:L - 1], v[:L - 1], qn, kn, shape, 1e-6, cache)
        return cache

    want = gdn_b200.attention_core(qg[L - 1:], k[L - 1:], v[L - 1:], qn, kn, shape, 1e-6, filled())
    cache = filled()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev())
    side.wait_stream(torch.cuda.current_stream(dev()))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            got = gdn_b200.attention_core(qg[L - 1:], k[L - 1:], v[L - 1:], qn, kn, shape, 1e-6, cache)
    torch.cuda.current_stream(dev()).wait_stream(side)
    for _ in range(2):  # the replay rewrites the same cache position
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    keys, _ = cache.state()
    assert cache.size == L and torch.isfinite(keys.float()).all()
    del graph
    gdn_b200.check_device_errors()


@pytest.mark.parametrize("heads,kv_heads,head_dim,rotary,cached",
                         [(8, 8, 64, 16, 300), (6, 2, 128, 32, 700), (16, 1, 128, 64, 200), (4, 1, 64, 16, 5200)])
def test_attention_bf16_decode_on_tensor_cores(heads, kv_heads, head_dim, rotary, cached):
    # one token against a cache filled on the GPU: the tensor-core decode
    # (query groups of 1, 3 and 16 rows; 5,200 cached positions give two
    # tiles per key split and splits past the end), against the oracle given
    # the same cached keys and values
    shape = AttentionShape(heads, kv_heads, head_dim, rotary, 1000000.0)
    hidden = 128
    rng = np.random.default_rng(heads * 100 + head_dim)
    w = _bf16_weights(_random_weights(rng, shape, hidden, 0.05))
    layer = _layer(w, shape, 1e-6, torch.bfloat16)
    cache = _cache(shape, max_context=cached + 4, dtype=torch.bfloat16)
    layer(t(O.bf16_round(rng.standard_normal((cached, hidden)).astype(np.float32)), torch.bfloat16), cache)
    for _ in range(2):
        keys, values = (n(a).astype(np.float64) for a in cache.state())
        x = O.bf16_round(rng.standard_normal((1, hidden)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        want, _, _ = O.attention_layer(x, w, keys, values, heads, kv_heads, head_dim, rotary, 1000000.0, 1e-6,
                                       rnd=O.bf16_round)
        assert O.rel_l2(n(got), want) < 1e-2, O.rel_l2(n(got), want)
    gdn_b200.check_device_errors()


def test_attention_bf16_long_prefill_at_model_shape():
    """16 query heads over 2 key/value heads of 256: a 600-token prefill
    (ten key tiles for the last query rows) and a 203-token chunk after it
    (queries at an offset that is not a tile multiple), against the oracle."""
    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    hidden, eps = 512, 1e-6
    rng = np.random.default_rng(23)
    w = _bf16_weights(_random_weights(rng, shape, hidden, 0.05))
    layer = _layer(w, shape, eps, torch.bfloat16)
    cache = _cache(shape, max_context=1024, dtype=torch.bfloat16)
    keys, values = np.zeros((2, 0, 256)), np.zeros((2, 0, 256))
    for L in (600, 203):
        x = O.bf16_round(rng.standard_normal((L, hidden)).astype(np.float32))
        got = layer(t(x, torch.bfloat16), cache)
        want, keys, values = O.attention_layer(x, w, keys, values, 16, 2, 256, 64, 10000000.0, eps,
                                               rnd=O.bf16_round)
        assert O.rel_l2(n(got), want) < 1e-2, (L, O.rel_l2(n(got), want))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_prefill_with_more_head_rows_than_one_prep_cta_covers(dtype):
    """40 query heads over 8 key/value heads of 128 (56 head rows per token):
    a prefill long enough that the prep kernel takes four rows per warp over
    eight warps (32 rows) and the other 24 one at a time, then a chunk at an
    offset that is not a tile multiple; bf16 (the tensor-core prefill) and
    float32 (the CUDA-core kernel) against the oracle."""
    shape = AttentionShape(40, 8, 128, 32, 1000000.0)
    hidden, eps = 256, 1e-6
    rng = np.random.default_rng(41)
    bf16 = dtype == torch.bfloat16
    w = _random_weights(rng, shape, hidden, 0.05)
    if bf16:
        w = _bf16_weights(w)
    layer = _layer(w, shape, eps, dtype)
    cache = _cache(shape, max_context=1024, dtype=dtype)
    keys, values = np.zeros((8, 0, 128)), np.zeros((8, 0, 128))
    for L in (400, 150):
        x = rng.standard_normal((L, hidden)).astype(np.float32)
        if bf16:
            x = O.bf16_round(x)
        got = layer(t(x, dtype), cache)
        want, keys, values = O.attention_layer(x, w, keys, values, 40, 8, 128, 32, 1000000.0, eps,
                                               **({"rnd": O.bf16_round} if bf16 else {}))
        assert O.rel_l2(n(got), want) < (1e-2 if bf16 else 1e-4), (L, O.rel_l2(n(got), want))
    assert cache.size == 550
