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


def _fused_worker(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    import gdn_b200
    from gdn_b200.sharding import GatheredHeads, all_gather_heads, head_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        # ragged length (2,000 = 31 chunks + 16 tokens), segmented single sequence
        T, hk, hv, d = 2000, 4, 8, 128
        g = torch.Generator(dev).manual_seed(11)
        q = torch.nn.functional.normalize(torch.randn(T, hk, d, device=dev, generator=g), dim=-1).bfloat16()
        k = torch.nn.functional.normalize(torch.randn(T, hk, d, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(T, hv, d, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(T, hv, device=dev, generator=g))
        gl = -torch.nn.functional.softplus(torch.randn(T, hv, device=dev, generator=g))
        ks, vs = head_shard(hk, hv, rank, world)
        ql, kl, vl = q[:, ks].contiguous(), k[:, ks].contiguous(), v[:, vs].contiguous()
        gll, bl = gl[:, vs].contiguous(), beta[:, vs].contiguous()
        res = []
        for dtype in (torch.float32, torch.bfloat16):
            y_loc, st_nccl = gdn_b200.gated_delta_scan_varlen(ql, kl, vl, gll, bl, None, g_is_log=True,
                                                              algo="chunked", out_dtype=dtype)
            y_nccl = all_gather_heads(y_loc, world)
            gh = GatheredHeads(T, hv, d, dtype, dev)
            for _ in range(2):  # twice: the second call overwrites the first's tiles everywhere
                gh.out.fill_(float("nan"))
                dist.barrier()
                y_fused, st_fused = gh.scan(ql, kl, vl, gll, bl, None, vs.start, g_is_log=True)
                torch.cuda.synchronize()
                res.append(bool(torch.equal(y_fused, y_nccl)) and bool(torch.equal(st_fused, st_nccl)))
            y_ref, _ = gdn_b200.gated_delta_scan_varlen(q, k, v, gl, beta, None, g_is_log=True, algo="chunked",
                                                        out_dtype=dtype)
            res.append(float((y_fused.float() - y_ref.float()).norm() / y_ref.float().norm()))
            gh.close()
        if rank == 0:
            np.save(path, np.array(res, dtype=np.float64))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_prefill_with_the_gather_fused_into_the_scan(tmp_path):
    """Each rank's scan writes its heads' output tiles into both ranks'
    gathered buffers over NVLink (gdn_scan_gathered): bit-identical to the
    NCCL all-gather of the same per-rank outputs, on two calls in a row, for
    float32 and bf16 outputs, and equal to the single-GPU scan."""
    path = str(tmp_path / "fused.npy")
    port = 29600 + (os.getpid() + 150) % 300
    mp.start_processes(_fused_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    r = np.load(path)
    # per dtype: [call 1 equal, call 2 equal, rel-L2 against one GPU]
    assert r[0] == 1 and r[1] == 1 and r[3] == 1 and r[4] == 1, r
    assert r[2] < 1e-5 and r[5] < 1e-5, r
