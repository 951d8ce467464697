"""Head sharding on 2 GPUs with NCCL: each rank runs the chunked prefill on
its GQA groups (value heads [r*Hv/2, (r+1)*Hv/2) with their key heads) and the
ranks all-gather the outputs; the gathered result must equal the single-GPU
result. Skipped when fewer than 2 GPUs are visible."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    import gdn_b200
    from gdn_b200.sharding import all_gather_heads, head_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        T, hk, hv, d = 700, 4, 8, 128
        g = torch.Generator(dev).manual_seed(7)
        q = torch.nn.functional.normalize(torch.randn(T, hk, d, device=dev, generator=g), dim=-1).bfloat16()
        k = torch.nn.functional.normalize(torch.randn(T, hk, d, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(T, hv, d, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(T, hv, device=dev, generator=g))
        gl = -torch.nn.functional.softplus(torch.randn(T, hv, device=dev, generator=g))
        ks, vs = head_shard(hk, hv, rank, world)
        y_loc, _ = gdn_b200.gated_delta_scan_varlen(q[:, ks].contiguous(), k[:, ks].contiguous(),
                                                    v[:, vs].contiguous(), gl[:, vs].contiguous(),
                                                    beta[:, vs].contiguous(), None, g_is_log=True, algo="chunked")
        y_all = all_gather_heads(y_loc, world)
        if rank == 0:
            y_ref, _ = gdn_b200.gated_delta_scan_varlen(q, k, v, gl, beta, None, g_is_log=True, algo="chunked")
            err = float((y_all - y_ref).norm() / y_ref.norm())
            np.save(path, np.array([err]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_prefill_with_nccl_all_gather(tmp_path):
    path = str(tmp_path / "err.npy")
    port = 29600 + os.getpid() % 300
    mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    err = float(np.load(path)[0])
    assert err < 1e-6, err  # identical kernels on identical per-head inputs
