"""The affine-quantized projection kernels (gdn_quantized_linear,
gdn_dequantize) against the oracle's restatement of mx.quantized_matmul
(model/moe_block.py:23-50): bf16 activations through the tcgen05 GEMM with
on-the-fly dequantization, float32 activations through the dequantized
weights, the reference test's own small shapes (hidden 128, group 64, 4 bits)
and the layer's projection shapes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200 import QuantScheme, dequantize, quantized_linear
from gpu_helpers import dev, n, t
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

# bf16 output: one rounding of an fp32 accumulation (rel-L2 about 1.1e-3
# against the exact product); against the bf16-rounded exact product the
# differences are the elements whose accumulation error crosses a rounding
# tie, a share that grows with k (tensor-core accumulation over K).
TOL_EXACT = 2e-3


def _tol_rounded(k):
    return 3e-4 * max(1.0, k / 2048) ** 0.5


def _weights(rng, nrows, k, bits, gs, biases=True, signed_scales=True):
    q = rng.integers(0, 1 << bits, size=(nrows, k))
    groups = k // gs
    s = rng.uniform(0.002, 0.02, size=(nrows, groups)).astype(np.float32)
    if signed_scales:
        s *= rng.choice([-1.0, 1.0], size=s.shape)
    s = O.bf16_round(s)
    b = O.bf16_round(rng.uniform(-0.1, 0.1, size=(nrows, groups)).astype(np.float32)) if biases else None
    return O.pack_affine(q, bits), s, b


def _torch_weights(words, s, b):
    out = {"weight": torch.from_numpy(words.view(np.int32)).to(dev()), "scales": t(s, torch.bfloat16)}
    if b is not None:
        out["biases"] = t(b, torch.bfloat16)
    return out


def _check(out, ref, k):
    got = n(out).astype(np.float64)
    assert np.isfinite(got).all()
    e1 = O.rel_l2(got, ref)
    e2 = O.rel_l2(got, O.bf16_round(ref.astype(np.float32)))
    assert e1 <= TOL_EXACT and e2 <= _tol_rounded(k), (e1, e2)


@pytest.mark.parametrize(
    "m,nn,k,bits,gs,biases",
    [
        (1, 32, 2048, 4, 64, True),        # one decode token, in_proj_a/b width (the GEMV)
        (1, 12352, 2048, 4, 64, True),     # one token through the fused in-projection width
        (3, 2048, 4096, 4, 64, True),      # out_proj, three tokens
        (8, 1000, 1088, 4, 32, False),     # eight tokens, k % 128 == 64
        (5, 777, 2048, 8, 64, True),       # 8-bit GEMV, ragged n
        (2, 64, 192, 8, 64, True),        # 8-bit, k % 128 == 64
        (3, 40, 64, 4, 64, True),          # k = 64: half the lanes of the only chunk are empty
        (1, 24, 64, 8, 32, False),
        (12, 520, 2048, 4, 64, True),      # two token blocks
        (16, 999, 1024, 8, 32, False),
        (16, 40, 6400, 4, 64, True),       # x staged near its size limit: 17 x 6400 x 2 bytes
        (16, 40, 8192, 4, 64, True),       # x too large to stage: the tiled GEMM
        (17, 300, 2048, 4, 128, True),     # from 17 tokens on: the tiled GEMM
        (32, 2048, 2048, 4, 64, True),
        (200, 700, 2048, 4, 64, True),
        (250, 300, 1024, 8, 64, True),
        (4, 4, 128, 4, 64, True),          # the reference test's in_proj_a shape
        (64, 256, 128, 4, 64, True),       # the reference test's in_proj_qkv shape
        (300, 999, 2048, 4, 64, True),     # ragged m and n (partial tiles, n % 8 != 0)
        (300, 1000, 1024, 4, 32, False),   # no biases
        (256, 640, 4096, 4, 128, True),
        (129, 520, 2048, 8, 64, True),
        (64, 256, 512, 8, 32, False),
        (512, 768, 1024, 8, 128, True),
        (4096, 1024, 2048, 4, 64, True),   # many tiles in both directions
    ],
)
def test_quantized_linear_bf16_matches_oracle(m, nn, k, bits, gs, biases):
    rng = np.random.default_rng(m * 7 + nn + k + bits)
    words, s, b = _weights(rng, nn, k, bits, gs, biases)
    x = O.bf16_round(rng.standard_normal((m, k)).astype(np.float32))
    out = quantized_linear(t(x, torch.bfloat16), _torch_weights(words, s, b), QuantScheme(bits=bits, group_size=gs))
    torch.cuda.synchronize()
    assert out.shape == (m, nn) and out.dtype == torch.bfloat16
    _check(out, O.quantized_linear_ref(x, words, s, b, bits, gs), k)
    gdn_b200.check_device_errors()


@pytest.mark.parametrize("bits,gs,biases", [(4, 64, True), (8, 32, True), (4, 128, False)])
def test_dequantize_is_bit_exact(bits, gs, biases):
    rng = np.random.default_rng(bits + gs)
    words, s, b = _weights(rng, 300, 1024, bits, gs, biases)
    w = _torch_weights(words, s, b)
    want = O.dequant_affine(words, s, b, bits, gs)
    q = QuantScheme(bits=bits, group_size=gs)
    np.testing.assert_array_equal(n(dequantize(w, q, torch.float32)), want)
    np.testing.assert_array_equal(n(dequantize(w, q, torch.bfloat16)), want)


def test_float32_activations_use_dequantized_weights():
    rng = np.random.default_rng(5)
    words, s, b = _weights(rng, 384, 1024, 4, 64)
    x = rng.standard_normal((70, 1024)).astype(np.float32)
    out = quantized_linear(t(x), _torch_weights(words, s, b), QuantScheme(bits=4, group_size=64))
    assert out.dtype == torch.float32
    ref = O.quantized_linear_ref(x, words, s, b, 4, 64)
    assert O.rel_l2(n(out), ref) <= 1e-5


def test_leading_dims_strided_rows_and_linear_weights():
    rng = np.random.default_rng(9)
    words, s, b = _weights(rng, 520, 2048, 4, 64)
    q = QuantScheme(bits=4, group_size=64)
    lw = gdn_b200.LinearWeights(_torch_weights(words, s, b), q)
    x = O.bf16_round(rng.standard_normal((2, 3, 80, 2048 + 64)).astype(np.float32))
    xt = t(x, torch.bfloat16)[..., 32:32 + 2048]  # rows with a stride of 2112 elements, 64-byte offset
    out = quantized_linear(xt, lw)
    assert out.shape == (2, 3, 80, 520)
    ref = O.quantized_linear_ref(x[..., 32:32 + 2048].reshape(-1, 2048), words, s, b, 4, 64)
    _check(out.reshape(-1, 520), ref, 2048)


def test_quantize_then_matmul_close_to_dense():
    # the reference tests' construction: quantize a dense weight, compare
    # with the plain product of its dequantized copy
    rng = np.random.default_rng(11)
    dense = rng.standard_normal((256, 128)).astype(np.float32) * 0.05
    words, s, b = O.quantize_affine(dense, 4, 64)
    x = O.bf16_round(rng.standard_normal((4, 128)).astype(np.float32))
    out = quantized_linear(t(x, torch.bfloat16), _torch_weights(words, s, b), QuantScheme(bits=4, group_size=64))
    eff = O.dequant_affine(words, s, b, 4, 64)
    _check(out, x.astype(np.float64) @ eff.astype(np.float64).T, 128)


def test_empty_batch():
    rng = np.random.default_rng(2)
    words, s, b = _weights(rng, 64, 128, 4, 64)
    out = quantized_linear(torch.empty(0, 128, device=dev(), dtype=torch.bfloat16), _torch_weights(words, s, b),
                           QuantScheme(bits=4, group_size=64))
    assert out.shape == (0, 64)
