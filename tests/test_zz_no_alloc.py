"""gdn_fused_block_noalloc: the fused block for callers that cannot allocate
device memory (a host driving the library through a plain C FFI with no device
allocator, where a cudaMalloc per call would synchronise the device, or a
server whose device memory is all reserved up front). It uses a fixed scratch
array compiled into the library instead of a caller workspace.

Checked through the C ABI against the allocating entry point
(gdn_fused_block) on two calls in a row with different inputs: both entry
points launch the same kernels on the same inputs, only the scratch address
differs, so the outputs must be bit-identical (the shared scratch keeps the
first call's contents, and any of it leaking into the second call would show).
The cases cover the token-serial path and the chunked tensor-core path, whose
records, tensor maps and segment buffers then live in the static scratch.
Collected last, so a run that stops at its first failure has run every other
test already."""

from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from gdn_b200 import _lib
from gdn_b200.linear_attention import LinearAttentionShape

SERIAL_SHAPE = LinearAttentionShape(2, 4, 64, 32, 4)     # head dims off the tensor-core path
CHUNKED_SHAPE = LinearAttentionShape(2, 4, 128, 128, 4)  # chunked path (128-dim heads, >= 128 tokens)


def _case(seed, lengths, dev, shape):
    rng = np.random.default_rng(seed)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    n_tok, n_seq = int(cu[-1]), len(lengths)
    t = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).to(dev, dt)
    return {
        "cu": t(cu, torch.int64),
        "mixed": t(rng.standard_normal((n_tok, shape.mixed_width)).astype(np.float32), torch.bfloat16),
        "conv_w": t((rng.standard_normal((shape.conv_dim, 4)) * 0.1).astype(np.float32)),
        "A_log": t(rng.uniform(0, 1.5, shape.num_value_heads).astype(np.float32)),
        "dt_bias": t((rng.standard_normal(shape.num_value_heads) * 0.1).astype(np.float32)),
        "norm_w": t((1 + 0.1 * rng.standard_normal(shape.value_head_dim)).astype(np.float32)),
        "conv_state": t(rng.standard_normal((n_seq, 3, shape.conv_dim)).astype(np.float32)),
        "ssm": t((rng.standard_normal((n_seq, shape.num_value_heads, shape.value_head_dim,
                                       shape.key_head_dim)) * 0.02).astype(np.float32)),
        "n_tok": n_tok,
        "n_seq": n_seq,
        "shape": shape,
    }


def _args(c, conv_out, ssm_out, out, workspace=None, nbytes=0):
    shape = c["shape"]
    a = _lib.BlockArgs()
    a.n_tokens, a.n_seqs, a.cu_seqlens = c["n_tok"], c["n_seq"], c["cu"].data_ptr()
    a.hk, a.hv = shape.num_key_heads, shape.num_value_heads
    a.dk, a.dv, a.conv_kernel = shape.key_head_dim, shape.value_head_dim, shape.conv_kernel_dim
    a.mixed, a.mixed_stride_t, a.act_dtype = c["mixed"].data_ptr(), shape.mixed_width, _lib.GDN_BF16
    a.conv_w = c["conv_w"].data_ptr()
    a.conv_state_in, a.conv_state_out = c["conv_state"].data_ptr(), conv_out.data_ptr()
    a.conv_state_dtype = _lib.GDN_F32
    a.A_log, a.dt_bias, a.norm_w, a.eps = c["A_log"].data_ptr(), c["dt_bias"].data_ptr(), c["norm_w"].data_ptr(), 1e-6
    a.state_in, a.state_out, a.out = c["ssm"].data_ptr(), ssm_out.data_ptr(), out.data_ptr()
    a.algo = _lib.GDN_ALGO_AUTO
    a.workspace, a.workspace_bytes = workspace, nbytes
    return a


def _run_both(c, lib, stream):
    shape = c["shape"]
    outs = {}
    for name in ("alloc", "noalloc"):
        conv_out = torch.empty_like(c["conv_state"])
        ssm_out = torch.empty_like(c["ssm"])
        out = torch.empty((c["n_tok"], shape.num_value_heads, shape.value_head_dim), dtype=torch.bfloat16,
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


@pytest.mark.gpu
@pytest.mark.parametrize("shape,cases", [
    (SERIAL_SHAPE, ((1, [37, 90, 5]), (2, [64, 1]))),
    (CHUNKED_SHAPE, ((3, [300, 129]), (4, [256]))),
], ids=["serial", "chunked"])
def test_noalloc_block_matches_the_allocating_entry_point_on_two_calls_in_a_row(shape, cases):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed, lengths in cases:
        c = _case(seed, lengths, dev, shape)
        outs = _run_both(c, lib, stream)
        for got, want in zip(outs["noalloc"], outs["alloc"]):
            assert torch.isfinite(got.float()).all()
            assert torch.equal(got, want)


# The rejection case passes made-up device addresses, so it runs in a child
# process that sees no GPU: were the size check ever to regress, the launch
# behind it would fail there with a CUDA error instead of touching a device.
_REJECT_CHILD = r"""
import ctypes, importlib.util, json, sys
spec = importlib.util.spec_from_file_location("gdn_lib", sys.argv[1])
L = importlib.util.module_from_spec(spec)
spec.loader.exec_module(L)
lib = L.load()
a = L.BlockArgs()
a.n_tokens, a.n_seqs = 1 << 20, 1
a.hk, a.hv, a.dk, a.dv, a.conv_kernel = 16, 32, 128, 128, 4
a.mixed, a.mixed_stride_t, a.act_dtype = 0x1000, 12352, L.GDN_BF16
a.conv_state_dtype = L.GDN_F32
a.conv_w = a.A_log = a.dt_bias = a.norm_w = 0x2000
a.state_out, a.conv_state_out, a.out, a.eps = 0x3000, 0x4000, 0x5000, 1e-6
st = lib.gdn_fused_block_noalloc(ctypes.byref(a), None)
print(json.dumps([st, lib.gdn_last_error().decode()]))
"""


def test_noalloc_block_rejects_calls_beyond_its_scratch():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", _REJECT_CHILD, os.path.join(os.path.dirname(_lib.__file__), "_lib.py")],
                         capture_output=True, text=True, env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    st, msg = json.loads(out.stdout.strip().splitlines()[-1])
    assert st == _lib.GDN_EUNSUPPORTED
    assert "static scratch" in msg and "fewer tokens" in msg
