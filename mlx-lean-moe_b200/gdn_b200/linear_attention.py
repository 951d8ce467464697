"""The gated-delta linear-attention block on B200.

``gated_delta_block`` is the fused part of the reference's
``Qwen3_5LinearAttention.__call__`` (``qw/linear_attention.py:103-124``, with
``qw/`` = ``src/mlx_lean_moe/model/qwen3_5/``): from the input projections
to the gated RMSNorm, as one call into libgdn_b200 (``gdn_fused_block``):
causal depthwise conv + SiLU, q/k rms-norm, forget gate and beta, the scan,
and ``silu(z) * rms_norm(y)``. The conv and ssm states are advanced in
place.

``Qwen3_5LinearAttention`` wraps it with the layer's projections
(``in_proj_qkv/z/b/a`` and ``out_proj``), dense or affine-quantized as the
reference's ``quantized_linear`` takes them (``model/moe_block.py:23-50``),
so the layer is a drop-in for the reference's class with a
``RecurrentCache``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .gated_delta import _DTYPES, _require_cuda, _stream
from .quantized import LinearWeights, QuantScheme, as_linear, concat_rows, quantized_linear
from .recurrent_cache import RecurrentCache


@dataclass(frozen=True)
class LinearAttentionShape:
    """``qw/config.py:10-32``: head counts/dims and conv kernel width."""

    num_key_heads: int
    num_value_heads: int
    key_head_dim: int
    value_head_dim: int
    conv_kernel_dim: int

    @property
    def key_dim(self) -> int:
        return self.num_key_heads * self.key_head_dim

    @property
    def value_dim(self) -> int:
        return self.num_value_heads * self.value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def mixed_width(self) -> int:
        """Row width of the mixed projection ``q | k | v | z | b | a``."""
        return self.conv_dim + self.value_dim + 2 * self.num_value_heads


def gated_delta_block(
    mixed: torch.Tensor,
    shape: LinearAttentionShape,
    conv_w: torch.Tensor,
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    norm_w: torch.Tensor,
    eps: float,
    conv_state: torch.Tensor | None,
    ssm_state: torch.Tensor,
    *,
    cu_seqlens: torch.Tensor | None = None,
    n_seqs: int | None = None,
    conv_state_out: torch.Tensor | None = None,
    ssm_state_out: torch.Tensor | None = None,
    algo: str = "auto",
    out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
    """Run the fused block over B packed sequences.

    ``mixed``: ``(N, W)`` float32 or bfloat16, rows ``q | k | v | z | b | a``.
    ``conv_w``: ``(C, K)`` or ``(C, K, 1)``. ``conv_state``: ``(B, K-1, C)``
    float32/bfloat16 or None (zeros); ``ssm_state``: float32 ``(B, Hv, Dv,
    Dk)``. Outputs default to in-place updates of the given states. Returns
    ``(out (N, Hv, Dv) in mixed's dtype, conv_state_out, ssm_state_out)``."""

    device = _require_cuda(mixed, conv_w, A_log, dt_bias, norm_w, conv_state, ssm_state, cu_seqlens)
    if mixed.ndim != 2 or mixed.shape[1] != shape.mixed_width or mixed.stride(1) != 1:
        raise ValueError(f"mixed must be (N, {shape.mixed_width}) with contiguous rows")
    if mixed.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("mixed must be float32 or bfloat16")
    if n_seqs is None:
        n_seqs = 1 if cu_seqlens is None else cu_seqlens.numel() - 1
    K = shape.conv_kernel_dim
    hv, dv, dk = shape.num_value_heads, shape.value_head_dim, shape.key_head_dim
    if tuple(ssm_state.shape) != (n_seqs, hv, dv, dk) or ssm_state.dtype != torch.float32:
        raise ValueError("ssm_state must be float32 (B, Hv, Dv, Dk)")
    if conv_state is not None and (tuple(conv_state.shape) != (n_seqs, K - 1, shape.conv_dim)
                                   or conv_state.dtype not in (torch.float32, torch.bfloat16)):
        raise ValueError("conv_state must be (B, K-1, conv_dim) float32 or bfloat16")
    conv_w2 = conv_w.reshape(shape.conv_dim, K).float().contiguous()
    A = A_log.float().contiguous()
    dt = dt_bias.float().contiguous()
    nw = norm_w.float().contiguous()
    ssm_in = ssm_state.contiguous()
    if ssm_state_out is None:
        ssm_state_out = ssm_in
    if conv_state_out is None and K > 1:
        conv_state_out = (conv_state if conv_state is not None
                          else torch.zeros((n_seqs, K - 1, shape.conv_dim), dtype=torch.float32, device=device))
    if out is None:
        out = torch.empty((mixed.shape[0], hv, dv), dtype=mixed.dtype, device=device)

    a = _lib.BlockArgs()
    a.n_tokens, a.n_seqs = mixed.shape[0], n_seqs
    a.cu_seqlens = cu_seqlens.data_ptr() if cu_seqlens is not None else None
    a.hk, a.hv, a.dk, a.dv, a.conv_kernel = shape.num_key_heads, hv, dk, dv, K
    a.mixed, a.mixed_stride_t, a.act_dtype = mixed.data_ptr(), mixed.stride(0), _DTYPES[mixed.dtype]
    a.conv_w = conv_w2.data_ptr()
    a.conv_state_in = conv_state.data_ptr() if conv_state is not None else None
    a.conv_state_out = conv_state_out.data_ptr() if conv_state_out is not None else None
    if K == 1:  # no conv history at all
        conv_state = conv_state_out = None
        a.conv_state_in = a.conv_state_out = None
    st_dtype = conv_state_out.dtype if conv_state_out is not None else torch.float32
    if conv_state is not None and conv_state.dtype != st_dtype:
        raise ValueError("conv_state and conv_state_out must share a dtype")
    a.conv_state_dtype = _DTYPES[st_dtype]
    a.A_log, a.dt_bias, a.norm_w, a.eps = A.data_ptr(), dt.data_ptr(), nw.data_ptr(), float(eps)
    a.state_in, a.state_out, a.out = ssm_in.data_ptr(), ssm_state_out.data_ptr(), out.data_ptr()
    a.algo = _lib.ALGOS[algo]
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.gdn_block_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)), "gated_delta_block")
        workspace = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=device)
        a.workspace, a.workspace_bytes = workspace.data_ptr(), nbytes.value
        _lib.check(lib.gdn_fused_block(ctypes.byref(a), _stream(device)), "gated_delta_block")
    return out, conv_state_out, ssm_state_out


class Qwen3_5LinearAttention:
    """``qw/linear_attention.py:35-127``.  Each projection is a dense
    ``(out, in)`` tensor, a ``LinearWeights``, or a ``{weight, scales,
    biases}`` dict stored with ``quant`` (the reference's
    ``config.other_quant``).  The four input projections run as one GEMM
    producing the mixed row q|k|v|z|b|a when they share a storage scheme;
    everything between the projections is one fused call.
    ``__call__(x, cache)`` takes ``(hidden,)`` for one decode step or
    ``(L, hidden)`` and returns the same rank, advancing ``cache``."""

    def __init__(
        self,
        shape: LinearAttentionShape,
        rms_norm_eps: float,
        in_proj_qkv,
        in_proj_z,
        in_proj_a,
        in_proj_b,
        conv1d_weight: torch.Tensor,
        A_log: torch.Tensor,
        dt_bias: torch.Tensor,
        norm_weight: torch.Tensor,
        out_proj,
        algo: str = "auto",
        quant: QuantScheme | None = None,
    ) -> None:
        self.shape = shape
        self.eps = rms_norm_eps
        parts = [as_linear(w, quant) for w in (in_proj_qkv, in_proj_z, in_proj_b, in_proj_a)]
        # One GEMM produces the mixed row q|k|v|z|b|a when the storage agrees.
        self.in_proj: LinearWeights | None = None
        self.in_parts = parts
        if len({p.quant for p in parts}) == 1:
            self.in_proj = concat_rows(parts)
        self.conv_w = conv1d_weight.reshape(shape.conv_dim, shape.conv_kernel_dim)
        self.A_log, self.dt_bias, self.norm_weight = A_log, dt_bias, norm_weight
        self.out_proj = as_linear(out_proj, quant)
        self.algo = algo

    def _mixed(self, rows: torch.Tensor) -> torch.Tensor:
        if self.in_proj is not None:
            mixed = quantized_linear(rows, self.in_proj)
        else:
            mixed = torch.cat([quantized_linear(rows, p) for p in self.in_parts], dim=-1)
        return mixed if mixed.stride(-1) == 1 and mixed.stride(0) % 8 == 0 else mixed.contiguous()

    def __call__(self, x: torch.Tensor, cache: RecurrentCache) -> torch.Tensor:
        if x.ndim not in (1, 2):
            raise ValueError(f"Qwen3_5LinearAttention expects 1-D or 2-D x, got shape {tuple(x.shape)}")
        squeeze = x.ndim == 1
        rows = x[None, :] if squeeze else x
        seq_len = rows.shape[0]
        mixed = self._mixed(rows)
        conv_state, ssm_state = cache.state()
        # the block writes every row of both new states when it has tokens, so
        # fresh buffers need no copy of the old ones (which stay as they were,
        # as with the reference's functional update)
        new_conv = torch.empty_like(conv_state) if seq_len else conv_state.clone()
        new_ssm = torch.empty_like(ssm_state) if seq_len else ssm_state.clone()
        out, _, _ = gated_delta_block(
            mixed, self.shape, self.conv_w, self.A_log, self.dt_bias, self.norm_weight, self.eps,
            conv_state[None], ssm_state[None], conv_state_out=new_conv[None], ssm_state_out=new_ssm[None],
            algo=self.algo,
        )
        cache.update(new_conv, new_ssm, advance=seq_len)
        result = quantized_linear(out.reshape(seq_len, -1), self.out_proj)
        return result[0] if squeeze else result
