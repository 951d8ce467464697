"""Torch-CPU port of the reference's ops path -- TEST/BENCH INFRASTRUCTURE.

This is what ``bench.py --impl reference`` and the ``cpu_baseline`` leg time:
the reference's CPU execution of the op is MLX's ops path
(``qw/gated_delta.py:93-109`` calling ``gated_delta_step`` ``:24-41``), a
loop over positions in which every step is a handful of whole-state array
operations. MLX is not installable here, so the same array program runs on
torch's CPU backend with every host thread. Same operation order as the
reference; float32 throughout, as the reference computes when the state is
float32. (qw/ = src/mlx_lean_moe/model/qwen3_5/ in the reference project.)
"""

from __future__ import annotations

import torch


def gated_delta_step(q, k, v, g, beta, state):
    """``qw/gated_delta.py:24-41``; q/k already repeated to the value heads."""
    state = state * g[:, None, None]
    read = (state * k[:, None, :]).sum(dim=-1)
    delta = (v - read) * beta[:, None]
    state = state + k[:, None, :] * delta[:, :, None]
    y = (state * q[:, None, :]).sum(dim=-1)
    return y, state


def gated_delta_scan_ops(q, k, v, g, beta, state):
    """``qw/gated_delta.py:93-109``: repeat-interleave GQA, then one step per
    position. ``g`` is the multiplicative decay. Single sequence."""
    repeat = v.shape[-2] // q.shape[-2]
    if repeat > 1:
        q = torch.repeat_interleave(q, repeat, dim=-2)
        k = torch.repeat_interleave(k, repeat, dim=-2)
    outputs = []
    for t in range(q.shape[0]):
        y, state = gated_delta_step(q[t], k[t], v[t], g[t], beta[t], state)
        outputs.append(y)
    return torch.stack(outputs), state
