"""Linear projections with affine-quantized weights: the layer's ``in_proj_*``
and ``out_proj`` (the reference's ``quantized_linear``,
``src/mlx_lean_moe/model/moe_block.py:23-50``, which calls
``mx.quantized_matmul``).

The weights keep the reference's storage: ``{"weight", "scales", "biases"}``
with ``weight`` the unsigned ``bits``-bit values packed into uint32 words
along the input dimension (value j of a word in bits ``[j * bits, (j + 1) *
bits)``), ``scales`` / ``biases`` one per ``group_size`` inputs, and
``W = scales * q + biases``.  bf16 activations run the fused tcgen05 kernel
(``gdn_quantized_linear``); float32 activations multiply the same weights,
dequantized by ``gdn_dequantize``, with a float32 GEMM.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

# The reference's accepted schemes (config.py:11-33): mode -> (bits, group sizes).
_SUPPORTED = {
    "affine": ({2, 3, 4, 5, 6, 8}, {32, 64, 128}),
    "mxfp4": ({4}, {32}),
    "mxfp8": ({8}, {32}),
    "nvfp4": ({4}, {16}),
}
# What this build's kernels run.
_RUNS = {"affine": ({4, 8}, {32, 64, 128})}


@dataclass(frozen=True)
class QuantScheme:
    """One quantization scheme (the reference's ``QuantScheme``, config.py:11-33)."""

    bits: int
    group_size: int
    mode: str = "affine"

    def __post_init__(self) -> None:
        if self.mode not in _SUPPORTED:
            raise ValueError(f"unsupported quantization mode {self.mode!r}")
        bits, groups = _SUPPORTED[self.mode]
        if self.bits not in bits or self.group_size not in groups:
            raise ValueError(
                f"unsupported {self.mode} quantization with bits={self.bits}, group_size={self.group_size}"
            )


@dataclass(frozen=True)
class LinearWeights:
    """A projection with its own storage scheme; ``quant`` is None for a dense matrix."""

    tensors: object
    quant: QuantScheme | None


def _check_runs(quant: QuantScheme) -> None:
    runs = _RUNS.get(quant.mode)
    if runs is None or quant.bits not in runs[0] or quant.group_size not in runs[1]:
        raise ValueError(
            f"quantized_linear: {quant.mode} with bits={quant.bits}, group_size={quant.group_size} "
            "has no kernel in this build (affine, bits 4 or 8)"
        )


def _args(x2d: torch.Tensor | None, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor | None,
          quant: QuantScheme, n: int, k: int, out: torch.Tensor | None) -> _lib.QLinearArgs:
    a = _lib.QLinearArgs()
    a.m = 0 if x2d is None else x2d.shape[0]
    a.n, a.k = n, k
    if x2d is not None:
        a.x, a.x_stride_m = x2d.data_ptr(), x2d.stride(0)
        a.out, a.out_stride_m = out.data_ptr(), out.stride(0)
    a.w = w.data_ptr()
    a.scales = scales.data_ptr()
    a.biases = biases.data_ptr() if biases is not None else None
    a.bits, a.group_size = quant.bits, quant.group_size
    return a


def _unpack(tensors: dict, quant: QuantScheme, x: torch.Tensor):
    w = tensors["weight"]
    scales = tensors["scales"]
    biases = tensors.get("biases")
    if w.dtype not in (torch.uint32, torch.int32) or w.dim() != 2:
        raise ValueError("quantized weight must be a 2-D uint32 (or int32) tensor")
    n = w.shape[0]
    k = w.shape[1] * 32 // quant.bits
    if scales.shape != (n, k // quant.group_size) or (biases is not None and biases.shape != scales.shape):
        raise ValueError(f"scales/biases must have shape {(n, k // quant.group_size)}")
    if scales.dtype != torch.bfloat16 or (biases is not None and biases.dtype != torch.bfloat16):
        raise ValueError("scales and biases must be bfloat16")
    for t in (w, scales, biases):
        if t is not None and (not t.is_cuda or t.device != x.device or not t.is_contiguous()):
            raise ValueError("weights must be contiguous CUDA tensors on x's device")
    return w, scales, biases, n, k


def dequantize(tensors: dict, quant: QuantScheme, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The dense [n, k] weights (each rounded to bf16, as the GEMM uses them)."""

    _check_runs(quant)
    w = tensors["weight"]
    if not w.is_cuda:
        raise ValueError("dequantize runs on CUDA tensors")
    w, scales, biases, n, k = _unpack(tensors, quant, w)
    dense = torch.empty(n, k, device=w.device, dtype=dtype)
    dt = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16}[dtype]
    a = _args(None, w, scales, biases, quant, n, k, None)
    lib = _lib.load()
    _lib.check(lib.gdn_dequantize(ctypes.byref(a), dt, dense.data_ptr(),
                                  ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)),
               "dequantize")
    return dense


def quantized_linear(x: torch.Tensor, tensors, quant: QuantScheme | None = None) -> torch.Tensor:
    """``x @ W^T`` for dense, or affine-quantized, weights (the reference's
    ``quantized_linear``).  ``x``: ``(..., k)`` on CUDA; returns ``(..., n)``
    in ``x``'s dtype."""

    if isinstance(tensors, LinearWeights):
        quant = tensors.quant
        tensors = tensors.tensors
    if isinstance(tensors, torch.Tensor):
        return x @ tensors.T
    if quant is None:
        raise ValueError("quantized linear weights require a quantization scheme")
    _check_runs(quant)
    if not x.is_cuda:
        raise ValueError("quantized_linear runs on CUDA tensors (no CPU path)")
    w, scales, biases, n, k = _unpack(tensors, quant, x)
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} features, the weights expect {k}")
    lead = x.shape[:-1]
    x2d = x.reshape(-1, k)
    if x.dtype == torch.float32:
        return (x2d @ dequantize(tensors, quant, torch.float32).T).reshape(*lead, n)
    if x.dtype != torch.bfloat16:
        raise ValueError("quantized_linear takes bfloat16 or float32 activations")
    if x2d.stride(-1) != 1 or x2d.stride(0) % 8 or x2d.data_ptr() % 16:
        x2d = x2d.contiguous()
    n_pad = (n + 7) // 8 * 8  # output rows padded to 16 bytes for the TMA store
    out = torch.empty(x2d.shape[0], n_pad, device=x.device, dtype=torch.bfloat16)
    if x2d.shape[0] > 0:
        a = _args(x2d, w, scales, biases, quant, n, k, out)
        lib = _lib.load()
        _lib.check(lib.gdn_quantized_linear(ctypes.byref(a),
                                            ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
                   "quantized_linear")
    return out[:, :n].reshape(*lead, n)


def as_linear(tensors, quant: QuantScheme | None = None) -> LinearWeights:
    """A projection as ``LinearWeights``: a dense tensor stays dense whatever
    ``quant`` says (the reference's rule, moe_block.py:33-36); a
    ``{weight, scales[, biases]}`` dict takes ``quant``."""

    if isinstance(tensors, LinearWeights):
        return tensors
    if isinstance(tensors, torch.Tensor):
        return LinearWeights(tensors, None)
    if isinstance(tensors, dict):
        if quant is None:
            raise ValueError("quantized linear weights require a quantization scheme")
        return LinearWeights(tensors, quant)
    raise TypeError(f"unsupported projection weights: {type(tensors).__name__}")


def concat_rows(parts: list[LinearWeights]) -> LinearWeights:
    """Stack projections that share a storage scheme along their output rows,
    so one GEMM computes all of them (the block's mixed row q|k|v|z|b|a).
    A part without biases contributes zero biases."""

    quants = {p.quant for p in parts}
    if len(quants) != 1:
        raise ValueError("concat_rows needs projections with one storage scheme")
    quant = quants.pop()
    if quant is None:
        return LinearWeights(torch.cat([p.tensors for p in parts], dim=0), None)
    ws = [p.tensors["weight"] for p in parts]
    if len({w.shape[1] for w in ws}) != 1:
        raise ValueError("concat_rows needs projections with the same input width")
    weight = torch.cat([w.view(torch.int32) for w in ws], dim=0)
    scales = torch.cat([p.tensors["scales"] for p in parts], dim=0)
    out = {"weight": weight, "scales": scales}
    if any(p.tensors.get("biases") is not None for p in parts):
        out["biases"] = torch.cat(
            [p.tensors["biases"] if p.tensors.get("biases") is not None else torch.zeros_like(p.tensors["scales"])
             for p in parts], dim=0)
    return LinearWeights(out, quant)
