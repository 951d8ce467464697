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


class GatheredHeads:
    """The gathered output of a head-sharded prefill, written by the scan
    itself: every rank holds a ``(N, Hv, Dv)`` buffer ``out``, and every other
    rank's buffer is mapped into this process (CUDA IPC over NVLink), so that
    :meth:`scan` writes this rank's value heads into all of them from the
    scan kernel's output stage (``gdn_scan_gathered``) instead of an
    all-gather after it. Collective: every rank of ``group`` constructs it
    with the same shape, and calls :meth:`scan` and :meth:`close` together."""

    def __init__(self, n_tokens: int, hv: int, dv: int, dtype: torch.dtype, device: torch.device, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self._lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world - 1 > _lib.MAX_GATHER_PEERS:
            raise ValueError(f"at most {_lib.MAX_GATHER_PEERS + 1} ranks")
        self.out = torch.empty((n_tokens, hv, dv), dtype=dtype, device=device)
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        offset = ctypes.c_uint64(0)
        with torch.cuda.device(device):
            _lib.check(self._lib.gdn_ipc_export(self.out.data_ptr(), handle, ctypes.byref(offset)), "gdn_ipc_export")
        mine = (self.rank, bytes(handle), offset.value)
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self._peers = []  # (address, offset) of the other ranks' buffers, mapped here
        with torch.cuda.device(device):
            for r, h, off in sorted(every):
                if r == self.rank:
                    continue
                hb = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
                ptr = ctypes.c_void_p(0)
                _lib.check(self._lib.gdn_ipc_import(hb, off, ctypes.byref(ptr)), "gdn_ipc_import")
                self._peers.append((ptr.value, off))
        self._flag = torch.zeros(1, device=device)

    def scan(self, q, k, v, g, beta, state, head0: int, *, g_is_log: bool = False, state_out=None,
             algo: str = "chunked"):
        """The chunked scan of this rank's heads ``[head0, head0 + v.shape[1])``
        (whole GQA groups, as :func:`head_shard` picks), its outputs written
        into every rank's ``out``; then a one-element all-reduce on the stream,
        after which ``out`` holds every rank's heads. Returns ``(out,
        state_out)``."""

        import ctypes

        import torch.distributed as dist

        from . import _lib
        from .gated_delta import _prepare_gates, _qkv_common, _inner_contiguous, _scan_args, _stream

        device = self.out.device
        n, hv = v.shape[0], v.shape[1]
        if n != self.out.shape[0] or v.shape[2] != self.out.shape[2] or not 0 <= head0 <= self.out.shape[1] - hv:
            raise ValueError("v must be (N, heads, Dv) with its heads inside the gathered output")
        q, k, v = _qkv_common(_inner_contiguous(q), _inner_contiguous(k), _inner_contiguous(v))
        g, beta = _prepare_gates(g, beta)
        if state_out is None:
            state_out = torch.empty((1, hv, v.shape[2], q.shape[2]), dtype=torch.float32, device=device)
        ga = _lib.GatherArgs()
        ga.hv_total, ga.head0, ga.n_peers = self.out.shape[1], head0, len(self._peers)
        for j, (ptr, _) in enumerate(self._peers):
            ga.peer_out[j] = ptr
        with torch.cuda.device(device):
            args = _scan_args(q, k, v, g, beta, state, state_out, self.out, 1, None, g_is_log, algo)
            ws_bytes = ctypes.c_size_t(0)
            _lib.check(self._lib.gdn_scan_workspace_size(ctypes.byref(args), ctypes.byref(ws_bytes)), "gathered scan")
            workspace = None
            if ws_bytes.value:
                workspace = torch.empty(ws_bytes.value, dtype=torch.uint8, device=device)
                args.workspace, args.workspace_bytes = workspace.data_ptr(), ws_bytes.value
            _lib.check(self._lib.gdn_scan_gathered(ctypes.byref(args), ctypes.byref(ga), _stream(device)),
                       "gathered scan")
            dist.all_reduce(self._flag, group=self.group)  # every rank's tiles have landed everywhere
        return self.out, state_out

    def close(self) -> None:
        """Unmaps the other ranks' buffers (every rank, after its last scan)."""

        import torch.distributed as dist

        from . import _lib

        dist.barrier(group=self.group)  # no rank still writes into a buffer being unmapped
        with torch.cuda.device(self.out.device):
            for ptr, off in self._peers:
                _lib.check(self._lib.gdn_ipc_release(ptr, off), "gdn_ipc_release")
        self._peers = []
