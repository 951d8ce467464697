"""Work partitioning across ranks (host logic), including a world-size-2
gloo run on CPU that shards by sequence and by value head, computes each
shard with the oracle and reassembles the result."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn_b200.sharding import all_gather_heads, cu_seqlens_of, head_shard, lpt_partition
from oracle import gdn_oracle as O


def test_lpt_partition_covers_every_sequence_once_and_balances():
    lengths = O.config5_lengths()
    assert int(lengths.sum()) == 516_496
    for n in (1, 2, 4, 8):
        parts = lpt_partition(lengths, n)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [int(lengths[p].sum()) for p in parts]
        # LPT bound: max load <= mean + longest job
        assert max(loads) <= sum(loads) / n + int(lengths.max())
        if n == 8:
            assert max(loads) / (sum(loads) / n) < 1.05


def test_lpt_is_deterministic_and_handles_more_parts_than_jobs():
    assert lpt_partition([5, 5, 5], 2) == [[0, 2], [1]]
    assert lpt_partition([3], 4) == [[0], [], [], []]
    with pytest.raises(ValueError):
        lpt_partition([1], 0)


def test_cu_seqlens_and_head_shards():
    assert cu_seqlens_of([3, 0, 2]) == [0, 3, 3, 5]
    k, v = head_shard(16, 32, 3, 8)
    assert (k.start, k.stop, v.start, v.stop) == (6, 8, 12, 16)
    # GQA group of value head h is key head h // 2: a shard keeps whole groups
    for h in range(v.start, v.stop):
        assert k.start <= h // 2 < k.stop
    with pytest.raises(ValueError):
        head_shard(16, 32, 0, 3)


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        lengths = [5, 9, 2, 7]
        n, hk, hv, dk, dv = sum(lengths), 2, 4, 16, 8
        q = O._l2n(rng.standard_normal((n, hk, dk))).astype(np.float32)
        k = O._l2n(rng.standard_normal((n, hk, dk))).astype(np.float32)
        v = rng.standard_normal((n, hv, dv)).astype(np.float32)
        g = rng.uniform(0.8, 1, (n, hv)).astype(np.float32)
        beta = rng.uniform(0, 1, (n, hv)).astype(np.float32)
        s0 = (rng.standard_normal((4, hv, dv, dk)) * 0.1).astype(np.float32)
        cu = np.array(cu_seqlens_of(lengths))
        # head sharding: this rank's GQA groups
        ks, vs = head_shard(hk, hv, rank, world)
        y_loc, _ = O.scan_varlen(q[:, ks], k[:, ks], v[:, vs], g[:, vs], beta[:, vs], cu, s0[:, vs])
        y_all = all_gather_heads(torch.from_numpy(y_loc.astype(np.float32)), world).numpy()
        # sequence sharding: LPT parts, no exchange; gather final states to compare
        part = lpt_partition(lengths, world)[rank]
        states = np.zeros_like(s0)
        for i in part:
            s, e = cu[i], cu[i + 1]
            _, st = O.scan_varlen(q[s:e], k[s:e], v[s:e], g[s:e], beta[s:e], np.array([0, e - s]), s0[i : i + 1])
            states[i] = st[0]
        total = torch.from_numpy(states)
        dist.all_reduce(total)  # each sequence is owned by exactly one rank
        if rank == 0:
            np.savez(result_path, y=y_all, states=total.numpy(), q=q, k=k, v=v, g=g, beta=beta, s0=s0, cu=cu)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding_reassembles_the_full_result(tmp_path):
    port = 29500 + os.getpid() % 1000
    path = str(tmp_path / "r.npz")
    mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    r = np.load(path)
    y, st = O.scan_varlen(r["q"], r["k"], r["v"], r["g"], r["beta"], r["cu"], r["s0"])
    np.testing.assert_allclose(r["y"], y, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(r["states"], st, rtol=1e-6, atol=1e-6)
