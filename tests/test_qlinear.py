"""Affine-quantized projections on the host: the packing format's known
answers, the oracle's dequantization, the scheme validation that mirrors the
reference's config (config.py:11-33) and the argument checks of the C entry
points (no GPU needed: every case fails before a launch)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gdn_b200 import QuantScheme, _lib, quantized_linear
from oracle import gdn_oracle as O


def test_pack_known_answers():
    # value j of a word sits in bits [j * bits, (j + 1) * bits)
    assert int(O.pack_affine(np.arange(8)[None, :], 4)[0, 0]) == 0x76543210
    assert int(O.pack_affine(np.array([[0x11, 0x22, 0x33, 0xFF]]), 8)[0, 0]) == 0xFF332211
    assert int(O.pack_affine(np.array([[15] + [0] * 7]), 4)[0, 0]) == 0xF


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_round_trip(bits):
    rng = np.random.default_rng(bits)
    q = rng.integers(0, 1 << bits, size=(7, 256))
    w = O.pack_affine(q, bits)
    assert w.dtype == np.uint32 and w.shape == (7, 256 * bits // 32)
    np.testing.assert_array_equal(O.unpack_affine(w, bits), q)
    with pytest.raises(ValueError):
        O.pack_affine(np.full((1, 8), 1 << bits), bits)


def test_dequant_is_scale_times_value_plus_bias():
    q = np.arange(64)[None, :] % 16
    w = O.pack_affine(q, 4)
    s = O.bf16_round(np.array([[0.5, 0.25]], np.float32))
    b = O.bf16_round(np.array([[-3.0, 1.0]], np.float32))
    d = O.dequant_affine(w, s, b, 4, 32)
    np.testing.assert_array_equal(d[0, :32], 0.5 * q[0, :32] - 3.0)
    np.testing.assert_array_equal(d[0, 32:], 0.25 * q[0, 32:] + 1.0)
    np.testing.assert_array_equal(O.dequant_affine(w, s, None, 4, 32)[0, :32], 0.5 * q[0, :32])


def test_dequant_rounds_to_nearest_even_bf16():
    # scale 2^-8, bias 1: every odd q lands on a tie between two bf16 values
    # (spacing 2^-7 above 1.0), which must go to the even one
    q = np.zeros((1, 32), np.int64)
    q[0, :4] = [1, 3, 5, 2]
    s = np.array([[2.0 ** -8]], np.float32)
    b = np.array([[1.0]], np.float32)
    d = O.dequant_affine(O.pack_affine(q, 4), s, b, 4, 32)
    assert d[0, 0] == np.float32(1.0)
    assert d[0, 1] == np.float32(1.0 + 2.0 ** -6)
    assert d[0, 2] == np.float32(1.0 + 2.0 ** -6)  # 1 + 5 * 2^-8: tie between 1 + 2^-6 and 1 + 3 * 2^-7
    assert d[0, 3] == np.float32(1.0 + 2.0 ** -7)  # exact


@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 32), (4, 128)])
def test_quantize_then_dequantize_is_close(bits, gs):
    rng = np.random.default_rng(1)
    dense = rng.standard_normal((16, 256)).astype(np.float32) * 0.05
    w, s, b = O.quantize_affine(dense, bits, gs)
    err = O.rel_l2(O.dequant_affine(w, s, b, bits, gs), dense)
    assert err < (0.12 if bits == 4 else 0.01)


def test_quant_scheme_validation_mirrors_reference():
    QuantScheme(bits=4, group_size=64)
    QuantScheme(bits=8, group_size=32, mode="mxfp8")
    QuantScheme(bits=4, group_size=16, mode="nvfp4")
    for bad in [dict(bits=7, group_size=64), dict(bits=4, group_size=48), dict(bits=4, group_size=32, mode="nf4"),
                dict(bits=8, group_size=32, mode="mxfp4")]:
        with pytest.raises(ValueError):
            QuantScheme(**bad)


def test_quantized_linear_host_behaviour():
    x = torch.randn(3, 64)
    dense = torch.randn(5, 64)
    torch.testing.assert_close(quantized_linear(x, dense), x @ dense.T)
    tensors = {"weight": torch.zeros(5, 8, dtype=torch.int32), "scales": torch.zeros(5, 1, dtype=torch.bfloat16)}
    with pytest.raises(ValueError, match="quantization scheme"):
        quantized_linear(x, tensors)
    with pytest.raises(ValueError, match="no kernel"):
        quantized_linear(x, tensors, QuantScheme(bits=2, group_size=64))
    with pytest.raises(ValueError, match="no CPU path"):
        quantized_linear(x, tensors, QuantScheme(bits=4, group_size=64))


def _args(**kw):
    a = _lib.QLinearArgs()
    a.m, a.n, a.k = 128, 256, 512
    a.x, a.x_stride_m, a.w, a.scales, a.out, a.out_stride_m = 0x1000, 512, 0x2000, 0x3000, 0x4000, 256
    a.bits, a.group_size = 4, 64
    for key, v in kw.items():
        setattr(a, key, v)
    return a


@pytest.mark.parametrize(
    "kw,fragment",
    [
        (dict(bits=3), "bits 4 and 8"),
        (dict(group_size=16), "group_size"),
        (dict(k=96), "multiple of 64"),
        (dict(k=64, group_size=128), "multiple of 64 and of group_size"),
        (dict(x_stride_m=100), "row strides"),
        (dict(out_stride_m=250), "row strides"),
        (dict(w=0x2004), "16-byte aligned"),
        (dict(scales=0), "non-NULL"),
        (dict(n=0), "n > 0"),
    ],
)
def test_quantized_linear_rejects_bad_arguments(kw, fragment):
    lib = _lib.load()
    st = lib.gdn_quantized_linear(ctypes.byref(_args(**kw)), None)
    assert st in (_lib.GDN_EINVAL, _lib.GDN_EUNSUPPORTED)
    assert fragment in lib.gdn_last_error().decode()


def test_dequantize_rejects_bad_arguments():
    lib = _lib.load()
    assert lib.gdn_quantized_linear(None, None) == _lib.GDN_EINVAL
    st = lib.gdn_dequantize(ctypes.byref(_args()), _lib.GDN_F16, 0x5000, None)
    assert st in (_lib.GDN_EINVAL, _lib.GDN_EUNSUPPORTED)
    assert lib.gdn_dequantize(ctypes.byref(_args()), _lib.GDN_F32, None, None) == _lib.GDN_EINVAL
    assert lib.gdn_dequantize(ctypes.byref(_args(bits=5)), _lib.GDN_F32, 0x5000, None) == _lib.GDN_EUNSUPPORTED


def test_as_linear_and_concat_rows_on_host():
    from gdn_b200 import LinearWeights, as_linear, concat_rows

    q4 = QuantScheme(bits=4, group_size=64)
    dense = torch.randn(3, 128)
    assert as_linear(dense, q4).quant is None  # a dense tensor stays dense
    with pytest.raises(ValueError, match="quantization scheme"):
        as_linear({"weight": torch.zeros(2, 16, dtype=torch.int32)})
    with pytest.raises(TypeError):
        as_linear([1, 2, 3])

    def part(rows, seed, biases=True):
        g = torch.Generator().manual_seed(seed)
        t = {"weight": torch.randint(0, 2**31 - 1, (rows, 16), dtype=torch.int32, generator=g),
             "scales": torch.rand(rows, 2, generator=g).bfloat16()}
        if biases:
            t["biases"] = torch.rand(rows, 2, generator=g).bfloat16()
        return LinearWeights(t, q4)

    a, b, c = part(5, 1), part(3, 2, biases=False), part(4, 3)
    cat = concat_rows([a, b, c])
    assert cat.quant == q4
    torch.testing.assert_close(cat.tensors["weight"], torch.cat([a.tensors["weight"], b.tensors["weight"],
                                                                  c.tensors["weight"]]))
    # the part without biases contributes zeros
    assert torch.all(cat.tensors["biases"][5:8] == 0)
    torch.testing.assert_close(cat.tensors["biases"][:5], a.tensors["biases"])
    d = concat_rows([LinearWeights(dense, None), LinearWeights(torch.randn(2, 128), None)])
    assert d.quant is None and d.tensors.shape == (5, 128)
    with pytest.raises(ValueError):
        concat_rows([a, LinearWeights(dense, None)])
