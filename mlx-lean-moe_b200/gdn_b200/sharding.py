"""Work partitioning across the GPUs of one node (one process per GPU).

The path shards without any data exchange: sequences are independent, and so
are value heads once each GQA group stays together (value heads
``[j*Hv/n, (j+1)*Hv/n)`` read key heads ``[j*Hk/n, (j+1)*Hk/n)``). The
only collective is the optional all-gather of head-sharded outputs.
"""

from __future__ import annotations

import heapq

import torch


def lpt_partition(lengths, n_parts: int) -> list[list[int]]:
    """Longest-processing-time bin packing: sequences in decreasing length
    order, each onto the currently least-loaded part (ties to the lowest
    part index). Returns the sequence indices of each part, each list in
    increasing index order. Deterministic for equal inputs."""

    if n_parts < 1:
        raise ValueError("n_parts must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, p) for p in range(n_parts)]
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        load, p = heapq.heappop(heap)
        parts[p].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), p))
    return [sorted(p) for p in parts]


def cu_seqlens_of(lengths) -> list[int]:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return cu


def head_shard(hk: int, hv: int, rank: int, world: int) -> tuple[slice, slice]:
    """Key-head and value-head slices owned by ``rank`` when value heads are
    split evenly over ``world`` ranks with GQA groups kept whole."""

    if hk % world or hv % world:
        raise ValueError(f"cannot split {hk} key / {hv} value heads over {world} ranks")
    kh, vh = hk // world, hv // world
    return slice(rank * kh, (rank + 1) * kh), slice(rank * vh, (rank + 1) * vh)


def all_gather_heads(local_out: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Gather head-sharded outputs ``(N, Hv/world, Dv)`` from every rank into
    ``(N, Hv, Dv)`` on every rank (one ``all_gather_into_tensor`` into a
    rank-major staging buffer, then a transpose into token-major order)."""

    import torch.distributed as dist

    n, hl, dv = local_out.shape
    staging = torch.empty((world, n, hl, dv), dtype=local_out.dtype, device=local_out.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(staging, local_out.contiguous(), group=group)
    else:  # gloo (CPU tests): list form
        dist.all_gather(list(staging.unbind(0)), local_out.contiguous(), group=group)
    return staging.permute(1, 0, 2, 3).reshape(n, world * hl, dv)
