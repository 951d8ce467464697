"""The C ABI: the library loads on a CPU-only host, exports every function
include/*.h declares (the operator interface gdn_api.h and the test hooks
gdn_testing.h), its ctypes structs match the C layout, and
argument errors come back as status codes before any CUDA call."""

from __future__ import annotations

import ctypes
import glob
import json
import os
import re
import subprocess
import sys

import pytest

from conftest import ROOT
from gdn_b200 import _lib

HEADER = os.path.join(ROOT, "include", "gdn_api.h")
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions() -> list[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names.update(re.findall(r"\b(gdn_[a-z_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    for name in names:
        assert re.search(rf"\bT {name}\b", out), f"{name} not exported"


def test_version():
    assert _lib.load().gdn_version() == 1


def _c_layout(tmp_path, struct: str, fields: list[str]) -> list[int]:
    src = tmp_path / "layout.c"
    lines = [f'#include "{HEADER}"', "#include <stdio.h>", "#include <stddef.h>", "int main(void){"]
    lines.append(f'printf("%zu\\n", sizeof({struct}));')
    for f in fields:
        lines.append(f'printf("%zu\\n", offsetof({struct}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    return [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]


@pytest.mark.parametrize("py,c", [(_lib.ScanArgs, "gdn_scan_args"), (_lib.DecodeArgs, "gdn_decode_args"),
                                  (_lib.BlockArgs, "gdn_block_args"), (_lib.QLinearArgs, "gdn_qlinear_args"),
                                  (_lib.AttnArgs, "gdn_attn_args"), (_lib.GatherArgs, "gdn_gather_args")])
def test_ctypes_structs_match_c_layout(tmp_path, py, c):
    fields = [f[0] for f in py._fields_]
    got = [ctypes.sizeof(py)] + [getattr(py, f).offset for f in fields]
    assert got == _c_layout(tmp_path, c, fields)


def _valid_args():
    a = _lib.ScanArgs()
    a.n_tokens, a.n_seqs = 4, 1
    a.hk, a.hv, a.dk, a.dv = 2, 4, 16, 8
    for name in ("q", "k", "v", "g", "beta", "out"):
        setattr(a, name, 0x1000)
    a.state_out = 0x2000
    return a


@pytest.mark.parametrize(
    "mutate,fragment",
    [
        (lambda a: setattr(a, "hv", 3), "multiple of its head count"),
        (lambda a: setattr(a, "dk", 0), "nonempty"),
        (lambda a: setattr(a, "n_seqs", 3), "multiple of n_seqs"),
        (lambda a: setattr(a, "state_out", 0x2004), "16-byte aligned"),
        (lambda a: setattr(a, "q", None), "non-NULL"),
        (lambda a: setattr(a, "q_stride_t", -1), "non-negative"),
        (lambda a: (setattr(a, "state_in", 0x2000 + 64)), "overlaps"),
        (lambda a: setattr(a, "out_dtype", _lib.GDN_F16), "out_dtype"),
        (lambda a: setattr(a, "dk", 18), "dk"),
        (lambda a: (setattr(a, "algo", _lib.GDN_ALGO_CHUNKED), setattr(a, "dk", 64)), "chunked"),
    ],
)
def test_scan_rejects_bad_arguments_on_the_host(mutate, fragment):
    lib = _lib.load()
    a = _valid_args()
    mutate(a)
    size = ctypes.c_size_t(0)
    st = lib.gdn_scan_workspace_size(ctypes.byref(a), ctypes.byref(size))
    assert st in (_lib.GDN_EINVAL, _lib.GDN_EUNSUPPORTED)
    assert fragment in lib.gdn_last_error().decode()


def test_null_args_and_decode_checks():
    lib = _lib.load()
    assert lib.gdn_scan(None, None) == _lib.GDN_EINVAL
    assert lib.gdn_decode(None, None) == _lib.GDN_EINVAL
    d = _lib.DecodeArgs()
    d.base = _valid_args()
    assert lib.gdn_decode(ctypes.byref(d), None) == _lib.GDN_EINVAL  # 4 tokens for 1 sequence
    assert "one token per sequence" in lib.gdn_last_error().decode()
    b = _lib.BlockArgs()
    assert lib.gdn_fused_block(ctypes.byref(b), None) == _lib.GDN_EINVAL
    assert lib.gdn_forget_gate(None, 0, 0, 4, 0, None, None, None, 0, None) == _lib.GDN_EINVAL


def test_block_workspace_size_is_host_only():
    lib = _lib.load()
    b = _lib.BlockArgs()
    b.n_tokens, b.n_seqs = 64, 2
    b.hk, b.hv, b.dk, b.dv, b.conv_kernel = 2, 4, 32, 32, 4
    b.mixed, b.mixed_stride_t = 0x1000, 2 * 64 + 2 * 128 + 8
    b.act_dtype, b.conv_state_dtype = _lib.GDN_BF16, _lib.GDN_F32
    b.conv_w = b.A_log = b.dt_bias = b.norm_w = 0x3000
    b.state_out, b.conv_state_out, b.out = 0x4000, 0x5000, 0x6000
    b.eps = 1e-6
    size = ctypes.c_size_t(0)
    assert lib.gdn_block_workspace_size(ctypes.byref(b), ctypes.byref(size)) == _lib.GDN_OK
    # q, k, v, y (bf16, the act dtype) + g, beta (fp32), each 256-byte aligned
    assert size.value >= 64 * (2 * 64 * 2 + 128 * 2 + 4 * 4 * 2 + 128 * 2)


def _attn_args(n_tokens=1, cache_len=4097):
    a = _lib.AttnArgs()
    a.n_tokens, a.cache_len, a.capacity = n_tokens, cache_len, max(cache_len, 4352)
    a.heads, a.kv_heads, a.head_dim, a.rotary_dim = 16, 2, 256, 64
    a.rope_base, a.eps, a.scale = 1e7, 1e-6, 256 ** -0.5
    a.qg, a.qg_stride_t = 0x10000, 16 * 512
    a.k_new, a.k_stride_t, a.v_new, a.v_stride_t = 0x20000, 512, 0x30000, 512
    a.q_norm = a.k_norm = 0x40000
    a.k_cache, a.v_cache = 0x50000, 0x60000
    a.act_dtype = _lib.GDN_BF16
    a.out, a.out_stride_t = 0x70000, 16 * 256
    return a


def _align256(x):
    return (x + 255) // 256 * 256


def test_attention_workspace_follows_the_split_rule():
    # one decode token: splits = min(2 x 148 CTAs over the row blocks, one
    # 32-key tile each, 160); the q rows, then the splits' partial rows
    # (head_dim + 4 floats each)
    lib = _lib.load()
    size = ctypes.c_size_t(0)
    assert lib.gdn_attention_workspace_size(ctypes.byref(_attn_args()), ctypes.byref(size)) == _lib.GDN_OK
    assert size.value == _align256(16 * 256 * 2) + _align256(129 * 16 * 260 * 4)  # 4,097 keys: 129 tiles
    assert lib.gdn_attention_workspace_size(ctypes.byref(_attn_args(1, 8000)), ctypes.byref(size)) == _lib.GDN_OK
    assert size.value == _align256(16 * 256 * 2) + _align256(148 * 16 * 260 * 4)  # 296 CTAs over 2 heads
    one_kv = _attn_args(1, 8000)
    one_kv.heads, one_kv.kv_heads = 8, 1
    assert lib.gdn_attention_workspace_size(ctypes.byref(one_kv), ctypes.byref(size)) == _lib.GDN_OK
    assert size.value == _align256(8 * 256 * 2) + _align256(160 * 8 * 260 * 4)  # capped at 160
    # a prefill of 4,096 tokens: one split, no partial rows
    assert lib.gdn_attention_workspace_size(ctypes.byref(_attn_args(4096, 4096)), ctypes.byref(size)) == _lib.GDN_OK
    assert size.value == _align256(4096 * 16 * 256 * 2)


# Rejection cases of gdn_attention as (field, value, message fragment).
_ATTN_BAD = [
    ("head_dim", 96, "head_dim"),
    ("rotary_dim", 63, "rotary_dim"),
    ("kv_heads", 3, "multiple of kv_heads"),
    ("cache_len", 0, "n_tokens <= cache_len"),
    ("k_cache", 0x50008, "16-byte aligned"),
    ("qg", None, "non-NULL"),
    ("act_dtype", _lib.GDN_F16, "float32 or bf16"),
    ("workspace_bytes", 64, "workspace too small"),
    ("workspace", 0x80008, "workspace must be 16-byte aligned"),
]

# The cases pass made-up device addresses, so they run in a child process
# that sees no GPU: if an argument check ever regressed, the launch behind it
# would fail there with a CUDA error instead of touching a device.
_ATTN_CHILD = r"""
import ctypes, importlib.util, json, sys
spec = importlib.util.spec_from_file_location("gdn_lib", sys.argv[1])
L = importlib.util.module_from_spec(spec)
spec.loader.exec_module(L)
lib = L.load()
cases = json.loads(sys.argv[2])
res = []
for field, value in cases:
    a = L.AttnArgs()
    a.n_tokens, a.cache_len, a.capacity = 1, 4097, 4352
    a.heads, a.kv_heads, a.head_dim, a.rotary_dim = 16, 2, 256, 64
    a.rope_base, a.eps, a.scale = 1e7, 1e-6, 256 ** -0.5
    a.qg, a.qg_stride_t = 0x10000, 16 * 512
    a.k_new, a.k_stride_t, a.v_new, a.v_stride_t = 0x20000, 512, 0x30000, 512
    a.q_norm = a.k_norm = 0x40000
    a.k_cache, a.v_cache = 0x50000, 0x60000
    a.act_dtype = L.GDN_BF16
    a.out, a.out_stride_t = 0x70000, 16 * 256
    size = ctypes.c_size_t(0)
    assert lib.gdn_attention_workspace_size(ctypes.byref(a), ctypes.byref(size)) == L.GDN_OK
    a.workspace, a.workspace_bytes = 0x80000, size.value
    setattr(a, field, value)
    st = lib.gdn_attention(ctypes.byref(a), None)
    res.append([st, lib.gdn_last_error().decode()])
print(json.dumps(res))
"""


@pytest.fixture(scope="module")
def attention_rejections():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cases = json.dumps([[f, v] for f, v, _ in _ATTN_BAD])
    out = subprocess.run([sys.executable, "-c", _ATTN_CHILD, os.path.join(os.path.dirname(_lib.__file__), "_lib.py"),
                          cases], capture_output=True, text=True, env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("case", range(len(_ATTN_BAD)), ids=[c[0] for c in _ATTN_BAD])
def test_attention_rejects_bad_arguments_before_any_launch(case, attention_rejections):
    st, msg = attention_rejections[case]
    assert st in (_lib.GDN_EINVAL, _lib.GDN_EUNSUPPORTED)
    assert _ATTN_BAD[case][2] in msg


# Rejection cases of gdn_scan_gathered as (field, value, message fragment);
# the scan arguments are valid ones at the model's head shape.
_GATHER_BAD = [
    ("head0", 17, "must lie in"),
    ("head0", -1, "must lie in"),
    ("hv_total", 8, "must lie in"),
    ("n_peers", 8, "n_peers"),
    ("reserved", 1, "reserved"),
    ("peer0", 0x90008, "16-byte aligned"),
    ("peer0", 0x70000, "other than out"),
    ("null", 0, "gather is NULL"),
]

# Made-up device addresses again, so the child sees no GPU (any launch a
# regressed check let through would fail with a CUDA error there).
_GATHER_CHILD = r"""
import ctypes, importlib.util, json, sys
spec = importlib.util.spec_from_file_location("gdn_lib", sys.argv[1])
L = importlib.util.module_from_spec(spec)
spec.loader.exec_module(L)
lib = L.load()
res = []
for field, value in json.loads(sys.argv[2]):
    a = L.ScanArgs()
    a.n_tokens, a.n_seqs = 4096, 1
    a.hk, a.hv, a.dk, a.dv = 8, 16, 128, 128
    a.q, a.q_stride_t, a.q_stride_h = 0x10000, 1024, 128
    a.k, a.k_stride_t, a.k_stride_h = 0x20000, 1024, 128
    a.v, a.v_stride_t, a.v_stride_h = 0x30000, 2048, 128
    a.g, a.g_stride_t, a.beta, a.beta_stride_t = 0x40000, 16, 0x50000, 16
    a.state_out, a.out = 0x60000, 0x70000
    a.qkv_dtype, a.gate_dtype, a.out_dtype = L.GDN_BF16, L.GDN_F32, L.GDN_BF16
    a.gate_kind, a.algo = L.GDN_GATE_LOG, L.GDN_ALGO_CHUNKED
    a.workspace, a.workspace_bytes = 0x80000, 1 << 40
    ga = L.GatherArgs()
    ga.hv_total, ga.head0, ga.n_peers = 32, 16, 1
    ga.peer_out[0] = 0x90000
    if field == "peer0":
        ga.peer_out[0] = value
    elif field != "null":
        setattr(ga, field, value)
    st = lib.gdn_scan_gathered(ctypes.byref(a), None if field == "null" else ctypes.byref(ga), None)
    res.append([st, lib.gdn_last_error().decode()])
print(json.dumps(res))
"""


@pytest.fixture(scope="module")
def gather_rejections():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cases = json.dumps([[f, v] for f, v, _ in _GATHER_BAD])
    out = subprocess.run([sys.executable, "-c", _GATHER_CHILD,
                          os.path.join(os.path.dirname(_lib.__file__), "_lib.py"), cases],
                         capture_output=True, text=True, env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("case", range(len(_GATHER_BAD)), ids=[f"{c[0]}={c[1]}" for c in _GATHER_BAD])
def test_gathered_scan_rejects_bad_gather_arguments_before_any_launch(case, gather_rejections):
    st, msg = gather_rejections[case]
    assert st == _lib.GDN_EINVAL, msg
    assert _GATHER_BAD[case][2] in msg
