"""gdn_fused_block_noalloc: the fused block for callers that cannot allocate
device memory (a host driving the library through a plain C FFI with no device
allocator, where a cudaMalloc per call would synchronise the device, or a
server whose device memory is all reserved up front). It uses a fixed scratch
array compiled into the library instead of a caller workspace.

Checked through the C ABI against the allocating entry point
(gdn_fused_block), within the tolerance the other block tests use, on two
calls in a row with different inputs (the shared scratch keeps the first
call's contents, which must not leak into the second). Collected last, so a
run that stops at its first failure has run every other test already."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gdn_b200 import _lib
from gdn_b200.linear_attention import LinearAttentionShape

pytestmark = pytest.mark.gpu

TOL = 2e-3  # rel-L2, as the bf16 block tests
SHAPE = LinearAttentionShape(2, 4, 64, 32, 4)


def _case(seed, lengths, dev):
    rng = np.random.default_rng(seed)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    n_tok, n_seq = int(cu[-1]), len(lengths)
    t = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).to(dev, dt)
    return {
        "cu": t(cu, torch.int64),
        "mixed": t(rng.standard_normal((n_tok, SHAPE.mixed_width)).astype(np.float32), torch.bfloat16),
        "conv_w": t((rng.standard_normal((SHAPE.conv_dim, 4)) * 0.1).astype(np.float32)),
        "A_log": t(rng.uniform(0, 1.5, SHAPE.num_value_heads).astype(np.float32)),
        "dt_bias": t((rng.standard_normal(SHAPE.num_value_heads) * 0.1).astype(np.float32)),
        "norm_w": t((1 + 0.1 * rng.standard_normal(SHAPE.value_head_dim)).astype(np.float32)),
        "conv_state": t(rng.standard_normal((n_seq, 3, SHAPE.conv_dim)).astype(np.float32)),
        "ssm": t((rng.standard_normal((n_seq, SHAPE.num_value_heads, SHAPE.value_head_dim,
                                       SHAPE.key_head_dim)) * 0.02).astype(np.float32)),
        "n_tok": n_tok,
        "n_seq": n_seq,
    }


def _args(c, conv_out, ssm_out, out, workspace=None, nbytes=0):
    a = _lib.BlockArgs()
    a.n_tokens, a.n_seqs, a.cu_seqlens = c["n_tok"], c["n_seq"], c["cu"].data_ptr()
    a.hk, a.hv = SHAPE.num_key_heads, SHAPE.num_value_heads
    a.dk, a.dv, a.conv_kernel = SHAPE.key_head_dim, SHAPE.value_head_dim, SHAPE.conv_kernel_dim
    a.mixed, a.mixed_stride_t, a.act_dtype = c["mixed"].data_ptr(), SHAPE.mixed_width, _lib.GDN_BF16
    a.conv_w = c["conv_w"].data_ptr()
    a.conv_state_in, a.conv_state_out = c["conv_state"].data_ptr(), conv_out.data_ptr()
    a.conv_state_dtype = _lib.GDN_F32
    a.A_log, a.dt_bias, a.norm_w, a.eps = c["A_log"].data_ptr(), c["dt_bias"].data_ptr(), c["norm_w"].data_ptr(), 1e-6
    a.state_in, a.state_out, a.out = c["ssm"].data_ptr(), ssm_out.data_ptr(), out.data_ptr()
    a.algo = _lib.GDN_ALGO_AUTO
    a.workspace, a.workspace_bytes = workspace, nbytes
    return a


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def _run_both(c, lib, stream):
    outs = {}
    for name in ("alloc", "noalloc"):
        conv_out = torch.empty_like(c["conv_state"])
        ssm_out = torch.empty_like(c["ssm"])
        out = torch.empty((c["n_tok"], SHAPE.num_value_heads, SHAPE.value_head_dim), dtype=torch.bfloat16,
                          device=c["mixed"].device)
        if name == "alloc":
            a = _args(c, conv_out, ssm_out, out)
            need = ctypes.c_size_t(0)
            _lib.check(lib.gdn_block_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace size")
            ws = torch.empty(need.value, dtype=torch.uint8, device=out.device)
            a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
            _lib.check(lib.gdn_fused_block(ctypes.byref(a), stream), "gdn_fused_block")
        else:
            a = _args(c, conv_out, ssm_out, out)  # no workspace given
            _lib.check(lib.gdn_fused_block_noalloc(ctypes.byref(a), stream), "gdn_fused_block_noalloc")
        torch.cuda.synchronize()
        outs[name] = (out, conv_out, ssm_out)
    return outs


def test_noalloc_block_matches_the_allocating_entry_point_on_two_calls_in_a_row():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed, lengths in ((1, [37, 90, 5]), (2, [64, 1])):
        c = _case(seed, lengths, dev)
        outs = _run_both(c, lib, stream)
        for got, want in zip(outs["noalloc"], outs["alloc"]):
            assert torch.isfinite(got.float()).all()
            assert _rel(got, want) <= TOL


def test_noalloc_block_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    a = _lib.BlockArgs()
    a.n_tokens, a.n_seqs = 1 << 20, 1
    a.hk, a.hv, a.dk, a.dv, a.conv_kernel = 16, 32, 128, 128, 4
    a.mixed, a.mixed_stride_t, a.act_dtype = 0x1000, 12352, _lib.GDN_BF16
    a.conv_state_dtype = _lib.GDN_F32
    a.conv_w = a.A_log = a.dt_bias = a.norm_w = 0x2000
    a.state_out, a.conv_state_out, a.out, a.eps = 0x3000, 0x4000, 0x5000, 1e-6
    st = lib.gdn_fused_block_noalloc(ctypes.byref(a), None)
    assert st == _lib.GDN_EUNSUPPORTED
    msg = lib.gdn_last_error().decode()
    assert "static scratch" in msg and "fewer tokens" in msg
