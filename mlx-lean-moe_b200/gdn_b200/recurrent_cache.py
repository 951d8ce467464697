"""Recurrent-state caches with the reference's layout, on the GPU.

``RecurrentCache`` mirrors ``src/mlx_lean_moe/cache/recurrent_cache.py:11-41``
of the reference: the last ``K - 1`` conv inputs ``(K-1, conv_dim)`` and the
float32 ssm state ``(Hv, Dv, Dk)``, Dk contiguous, with ``state()`` and
``update()``. ``BatchedRecurrentCache`` stacks B of them on a leading axis,
the layout the batched kernels read and update in place.
"""

from __future__ import annotations

import torch


class RecurrentCache:
    """One gated-delta layer's rolling state (single sequence)."""

    def __init__(
        self,
        conv_kernel_dim: int,
        conv_dim: int,
        num_value_heads: int,
        value_head_dim: int,
        key_head_dim: int,
        dtype: torch.dtype = torch.float32,
        device: torch.device | str = "cuda",
    ) -> None:
        if conv_kernel_dim < 1:
            raise ValueError(f"conv_kernel_dim must be positive, got {conv_kernel_dim}")
        self.conv_state = torch.zeros((conv_kernel_dim - 1, conv_dim), dtype=dtype, device=device)
        # float32 whatever the activation dtype: it accumulates over the whole
        # sequence (recurrent_cache.py:28-32).
        self.ssm_state = torch.zeros(
            (num_value_heads, value_head_dim, key_head_dim), dtype=torch.float32, device=device
        )
        self.size = 0

    def state(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.conv_state, self.ssm_state

    def update(self, conv_state: torch.Tensor, ssm_state: torch.Tensor, advance: int) -> None:
        self.conv_state = conv_state
        self.ssm_state = ssm_state
        self.size += advance


class BatchedRecurrentCache:
    """B sequences' states: conv ``(B, K-1, conv_dim)``, ssm float32
    ``(B, Hv, Dv, Dk)``, and per-sequence token counts. Kernels update both
    in place."""

    def __init__(
        self,
        batch: int,
        conv_kernel_dim: int,
        conv_dim: int,
        num_value_heads: int,
        value_head_dim: int,
        key_head_dim: int,
        dtype: torch.dtype = torch.float32,
        device: torch.device | str = "cuda",
    ) -> None:
        if conv_kernel_dim < 1:
            raise ValueError(f"conv_kernel_dim must be positive, got {conv_kernel_dim}")
        if batch < 1:
            raise ValueError(f"batch must be positive, got {batch}")
        self.conv_state = torch.zeros((batch, conv_kernel_dim - 1, conv_dim), dtype=dtype, device=device)
        self.ssm_state = torch.zeros(
            (batch, num_value_heads, value_head_dim, key_head_dim), dtype=torch.float32, device=device
        )
        self.sizes = [0] * batch

    def state(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.conv_state, self.ssm_state

    def advance(self, lengths) -> None:
        for i, n in enumerate(lengths):
            self.sizes[i] += int(n)
