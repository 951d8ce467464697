"""Error path and host-thread safety of the chunked prefill.

* A bounded device wait that runs out: with the wait limit cut to 1 ms and a
  test fault that withholds one V tile (so the barrier the state-chain warps
  wait on is never completed), the scan must give up, drain its own copies and
  MMAs, free its tensor memory and return; gdn_check_device_errors must report
  GDN_ETIMEOUT, and a normal call afterwards must match the oracle.  No kernel
  waits without a limit and nothing faults: the failure is a barrier that
  nothing completes.
* Two host threads, each on its own stream, running the time-segmented
  single-sequence scan (which forks work to a per-device side stream) on
  inputs that each thread writes on its own stream just before the call: the
  results must equal those of one thread alone, bit for bit.
* One process driving two GPUs: the chunked fused block and the attention
  prefill on cuda:0, then on cuda:1 (each device needs its own
  shared-memory opt-in); skipped with fewer than two GPUs.
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200 import _lib
from gpu_helpers import n, t
from oracle import gdn_oracle as O
from oracle import oracle_c

pytestmark = pytest.mark.gpu
DESIGN = 1e-3  # rel-L2 the chunked tests hold the tensor-core path to


def _prefill(lengths, hk, hv, seed):
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    q, k, v, g_log, beta = O.prefill_inputs(seed, int(cu[-1]), hk, hv, 128, 128)
    q, k, v = O.bf16_round(q), O.bf16_round(k), O.bf16_round(v)
    s0 = (np.random.default_rng(seed + 1).standard_normal((len(lengths), hv, 128, 128)) * 0.02).astype(np.float32)
    return q, k, v, g_log, beta, cu, s0


def _scan(q, k, v, g, beta, cu, s0):
    return gdn_b200.gated_delta_scan_varlen(
        t(q, torch.bfloat16), t(k, torch.bfloat16), t(v, torch.bfloat16), t(g), t(beta), t(s0),
        t(cu, torch.int64), g_is_log=True, algo="chunked")


def test_a_wait_that_runs_out_reports_timeout_and_the_next_call_is_correct():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    q, k, v, g, beta, cu, s0 = _prefill([200, 130], 2, 4, seed=11)
    assert lib.gdn_check_device_errors(stream) == _lib.GDN_OK  # nothing pending from earlier tests
    try:
        _lib.check(lib.gdn_test_set_wait_limit(1_000_000), "wait limit")  # 1 ms
        _lib.check(lib.gdn_test_inject_fault(1), "inject fault")
        _scan(q, k, v, g, beta, cu, s0)
        st = lib.gdn_check_device_errors(stream)
        msg = lib.gdn_last_error().decode()
    finally:
        _lib.check(lib.gdn_test_inject_fault(0), "clear fault")
        _lib.check(lib.gdn_test_set_wait_limit(0), "default wait limit")
    assert st == _lib.GDN_ETIMEOUT, (st, msg)
    assert "bounded device wait" in msg
    assert lib.gdn_check_device_errors(stream) == _lib.GDN_OK  # reported once, then cleared
    # the context is intact and the next call is correct
    y, s = _scan(q, k, v, g, beta, cu, s0)
    assert lib.gdn_check_device_errors(stream) == _lib.GDN_OK
    ey, es = oracle_c.scan_varlen(q, k, v, g, beta, cu, s0, g_is_log=True)
    assert O.rel_l2(n(y), ey) <= DESIGN
    assert O.rel_l2(n(s), es) <= DESIGN


def test_hook_arguments_are_checked():
    lib = _lib.load()
    assert lib.gdn_test_inject_fault(7) == _lib.GDN_EINVAL
    assert lib.gdn_test_inject_fault(-1) == _lib.GDN_EINVAL


def test_two_host_threads_run_segmented_scans_on_their_own_streams():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, hk, hv = 4096, 4, 8  # one dense sequence of 64 chunks: eight time segments, side-stream prep
    srcs = []
    for seed in (21, 22):
        q, k, v, g, beta, _, _ = _prefill([T], hk, hv, seed)
        srcs.append(tuple(t(x, dt) for x, dt in ((q, torch.bfloat16), (k, torch.bfloat16), (v, torch.bfloat16),
                                                 (g, torch.float32), (beta, torch.float32))))
    torch.cuda.synchronize()

    def run(bufs, src, stream):
        with torch.cuda.stream(stream):
            for b, x in zip(bufs, src):
                b.copy_(x, non_blocking=True)  # this thread's inputs, written on its own stream
            y, s = gdn_b200.gated_delta_scan_varlen(*bufs, None, g_is_log=True, algo="chunked")
        return y, s

    # one thread alone: the expected bits for each input
    alone = []
    for src in srcs:
        bufs = [torch.empty_like(x) for x in src]
        s = torch.cuda.Stream(dev)
        y, st = run(bufs, src, s)
        s.synchronize()
        alone.append((y.clone(), st.clone()))

    results = [None, None]
    errors = []

    def worker(i):
        try:
            torch.cuda.set_device(dev)
            s = torch.cuda.Stream(dev)
            bufs = [torch.empty_like(x) for x in srcs[0]]
            for rep in range(8):  # alternate the inputs; the last one is srcs[i]
                y, st = run(bufs, srcs[(i + rep + 1) % 2], s)
            s.synchronize()
            results[i] = (y, st)
        except Exception as e:  # reported on the main thread
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    assert _lib.load().gdn_check_device_errors(None) == _lib.GDN_OK
    for i in range(2):
        assert torch.equal(results[i][0], alone[i][0])
        assert torch.equal(results[i][1], alone[i][1])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_one_process_drives_two_gpus():
    from gdn_b200 import AttentionShape, GrowingKVCache
    from gdn_b200.linear_attention import LinearAttentionShape

    shape = LinearAttentionShape(2, 4, 128, 128, 4)
    rng = np.random.default_rng(5)
    mixed = O.bf16_round(rng.standard_normal((300, shape.mixed_width)).astype(np.float32))
    conv_w = (rng.standard_normal((shape.conv_dim, 4)) * 0.1).astype(np.float32)
    A_log = rng.uniform(0, 1.5, 4).astype(np.float32)
    dt_bias = (rng.standard_normal(4) * 0.1).astype(np.float32)
    norm_w = np.ones(128, np.float32)
    ashape = AttentionShape(16, 2, 256, 64, 10000000.0)
    qg = rng.standard_normal((512, 16 * 512)).astype(np.float32)
    kk = rng.standard_normal((512, 2 * 256)).astype(np.float32)
    vv = rng.standard_normal((512, 2 * 256)).astype(np.float32)
    got = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            T = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).to(dev, dt)
            cs = torch.zeros(1, 3, shape.conv_dim, device=dev)
            ss = torch.zeros(1, 4, 128, 128, device=dev)
            out, _, _ = gdn_b200.gated_delta_block(T(mixed, torch.bfloat16), shape, T(conv_w), T(A_log),
                                                   T(dt_bias), T(norm_w), 1e-6, cs, ss, algo="chunked")
            cache = GrowingKVCache(600, 2, 256, dtype=torch.bfloat16, device=dev)
            qn = torch.ones(256, device=dev)
            att = gdn_b200.attention_core(T(qg, torch.bfloat16), T(kk, torch.bfloat16), T(vv, torch.bfloat16),
                                          qn, qn, ashape, 1e-6, cache)
            torch.cuda.synchronize(dev)
            got.append([x.cpu() for x in (out, ss, att)])
    for a, b in zip(got[0], got[1]):
        assert torch.equal(a, b)
