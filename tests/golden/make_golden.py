"""Generate the golden vectors that pin the oracle to the reference.

Run where the reference project is checked out (read-only), with
``REFERENCE_ROOT`` set to that checkout::

    REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py

It writes ``golden.npz`` (outputs) and ``golden_manifest.json`` (sha256 of
every input array, so tests can regenerate the inputs from their seeds and
prove they are the same bytes). What it runs:

* the reference's own test generator ``_inputs`` and float64 recurrence
  ``_reference`` from ``tests/test_gated_delta_metal.py:10-39``, extracted
  from the test file with ``ast`` and executed as written (their only MLX
  use, ``mx.array``, becomes ``np.asarray``);
* the reference's own modules ``qw/gated_delta.py``,
  ``qw/linear_attention.py``, ``cache/recurrent_cache.py``, ``qw/attention.py``,
  ``model/rope.py`` and ``cache/kv_cache.py``, imported
  unchanged on the numpy MLX stand-in of ``mlx_numpy_shim.py`` (no Metal, so
  ``gated_delta_scan`` takes its ops path ``qw/gated_delta.py:93-109``).

``qw/`` is ``src/mlx_lean_moe/model/qwen3_5/`` in the reference project.
Nothing at test time reads the reference tree: tests load the committed
files only.
"""

from __future__ import annotations

import ast
import hashlib
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", "")

# Shapes of tests/test_gated_delta_metal.py:42-45, (L, Dk, Dv, Hk, Hv).
METAL_SHAPES = [(1, 32, 5, 3, 6), (7, 64, 32, 2, 2), (17, 128, 128, 16, 32), (129, 256, 7, 2, 6)]
LONG_LENGTH = 2048
# Layer test shapes of tests/test_qwen3_5_linear_attention.py:20-29.
LAYER = dict(hidden=128, hk=2, hv=4, dk=32, dv=32, kernel=4, eps=1e-6)
# Attention test shapes of tests/test_qwen3_5_attention.py:20-27.
ATTN = dict(hidden=128, heads=4, kv_heads=2, head_dim=32, rotary=8, theta=10000000.0, eps=1e-6)
# (seed, seq_len) cases of tests/test_qwen3_5_gated_delta.py.
GDN_CASES = [(0, 1), (0, 5), (1, 5), (2, 1), (3, 4)]


def sha(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def metal_key(shape) -> str:
    return "metal_" + "_".join(str(s) for s in shape)


def layer_case(seed: int, x_seed: int, seq_len: int):
    """Weights and input for one layer case, drawn in the order of
    ``_build_pair`` (``tests/test_qwen3_5_linear_attention.py:72-91``) but kept
    dense (the reference's quantize/dequantize round trip is an MLX call the
    stand-in does not provide): in_proj_qkv, in_proj_z, in_proj_a, in_proj_b,
    out_proj ~ 0.05 N(0,1); conv weight ~ 0.2 N(0,1) ``(C, K, 1)``; A_log,
    dt_bias ~ N(0,1); norm weight ~ 1 + 0.1 N(0,1). x ~ N(0,1) from
    ``default_rng(x_seed)``."""

    hidden, hk, hv, dk, dv, kernel = (LAYER[k] for k in ("hidden", "hk", "hv", "dk", "dv", "kernel"))
    key_dim, value_dim = hk * dk, hv * dv
    conv_dim = 2 * key_dim + value_dim
    rng = np.random.default_rng(seed)

    def dense(out_dim, in_dim):
        return (rng.standard_normal((out_dim, in_dim)).astype(np.float32) * 0.05).astype(np.float32)

    w = {}
    w["in_proj_qkv"] = dense(conv_dim, hidden)
    w["in_proj_z"] = dense(value_dim, hidden)
    w["in_proj_a"] = dense(hv, hidden)
    w["in_proj_b"] = dense(hv, hidden)
    w["out_proj"] = dense(hidden, value_dim)
    w["conv1d_weight"] = (rng.standard_normal((conv_dim, kernel, 1)).astype(np.float32) * 0.2).astype(np.float32)
    w["A_log"] = rng.standard_normal(hv).astype(np.float32)
    w["dt_bias"] = rng.standard_normal(hv).astype(np.float32)
    w["norm_weight"] = (rng.standard_normal(dv).astype(np.float32) * 0.1 + 1.0).astype(np.float32)
    x = np.random.default_rng(x_seed).standard_normal((seq_len, hidden)).astype(np.float32)
    return w, x


def attn_case(seed: int):
    """Dense weights of one attention case, drawn in the order of
    ``_build_pair`` (``tests/test_qwen3_5_attention.py:74-86``): q_proj (queries
    and gate, 2 x heads x head_dim rows), k_proj, v_proj, o_proj ~ 0.05 N(0,1);
    q_norm, k_norm ~ 1 + 0.1 N(0,1)."""

    h, hkv, hd, hidden = ATTN["heads"], ATTN["kv_heads"], ATTN["head_dim"], ATTN["hidden"]
    rng = np.random.default_rng(seed)

    def dense(out_dim, in_dim):
        return (rng.standard_normal((out_dim, in_dim)).astype(np.float32) * 0.05).astype(np.float32)

    w = {"q_proj": dense(h * hd * 2, hidden), "k_proj": dense(hkv * hd, hidden), "v_proj": dense(hkv * hd, hidden),
         "o_proj": dense(hidden, h * hd)}
    w["q_norm"] = (rng.standard_normal(hd).astype(np.float32) * 0.1 + 1.0).astype(np.float32)
    w["k_norm"] = (rng.standard_normal(hd).astype(np.float32) * 0.1 + 1.0).astype(np.float32)
    return w


def _extract_functions(path: str, names: list[str], namespace: dict) -> dict:
    source = open(path).read()
    tree = ast.parse(source)
    wanted = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    module = ast.Module(body=wanted, type_ignores=[])
    exec(compile(module, path, "exec"), namespace)
    return {n: namespace[n] for n in names}


def main() -> None:
    if not REFERENCE_ROOT:
        raise SystemExit("set REFERENCE_ROOT to the reference project's checkout")
    sys.path.insert(0, HERE)
    import mlx_numpy_shim

    refmods = mlx_numpy_shim.load_reference_modules(f"{REFERENCE_ROOT}/src")
    gd = refmods["gated_delta"]
    la = refmods["linear_attention"]
    rc = refmods["recurrent_cache"]
    qc = refmods["qconfig"]
    cfg = refmods["config"]

    mx_stub = types.SimpleNamespace(array=np.asarray)
    metal = _extract_functions(
        f"{REFERENCE_ROOT}/tests/test_gated_delta_metal.py",
        ["_inputs", "_reference"],
        {"np": np, "mx": mx_stub},
    )
    gdn_inputs = _extract_functions(
        f"{REFERENCE_ROOT}/tests/test_qwen3_5_gated_delta.py",
        ["_inputs"],
        {"np": np, "mx": mx_stub, "HK": 2, "HV": 6, "DK": 16, "DV": 8},
    )["_inputs"]

    arrays: dict[str, np.ndarray] = {}
    manifest: dict[str, dict] = {"inputs": {}, "source": {
        "generator": "tests/test_gated_delta_metal.py:10-39 (_inputs, _reference) executed as written",
        "op": "qw/gated_delta.py (ops path) on the numpy MLX stand-in",
        "layer": "qw/linear_attention.py Qwen3_5LinearAttention with dense projections",
    }}

    # 1. The Metal known-answer shapes.
    for shape in METAL_SHAPES:
        key = metal_key(shape)
        inputs = [np.asarray(a) for a in metal["_inputs"](*shape)]
        expected_y, expected_state = metal["_reference"](inputs)
        # The reference's own ops path agrees with its float64 recurrence.
        ref_y, ref_state = gd.gated_delta_scan(*inputs)
        np.testing.assert_allclose(ref_y, expected_y, rtol=2e-5, atol=2e-6)
        np.testing.assert_allclose(ref_state, expected_state, rtol=2e-5, atol=2e-6)
        manifest["inputs"][key] = [sha(a) for a in inputs]
        arrays[f"{key}/y"] = expected_y.astype(np.float32)
        if expected_state.size > 100_000:
            # Large state: every 4th value head plus whole-state checksums.
            arrays[f"{key}/state_heads_every4"] = expected_state[::4].astype(np.float32)
            arrays[f"{key}/state_sum"] = np.array(expected_state.sum())
            arrays[f"{key}/state_sumsq"] = np.array((expected_state**2).sum())
        else:
            arrays[f"{key}/state"] = expected_state.astype(np.float32)

    # 2. The long scan (tests/test_gated_delta_metal.py:74-98).
    inputs = [np.asarray(a) for a in metal["_inputs"](LONG_LENGTH)]
    expected_y, expected_state = metal["_reference"](inputs)
    manifest["inputs"]["long"] = [sha(a) for a in inputs]
    arrays["long/y_every8"] = expected_y[::8].astype(np.float32)
    arrays["long/y_sum"] = np.array(expected_y.sum())
    arrays["long/state"] = expected_state.astype(np.float32)

    # 3. Gates and scan of tests/test_qwen3_5_gated_delta.py, through the
    #    reference's forget_gate / sigmoid / gated_delta_scan.
    for seed, seq_len in GDN_CASES:
        key = f"gdn_{seed}_{seq_len}"
        x = {k: np.asarray(v) for k, v in gdn_inputs(seed, seq_len).items()}
        manifest["inputs"][key] = {k: sha(v) for k, v in x.items()}
        g = gd.forget_gate(x["a"], x["A_log"], x["dt_bias"])
        beta = la.mx.sigmoid(x["b"])
        state = np.zeros((6, 8, 16), np.float32)
        y, new_state = gd.gated_delta_scan(x["q"], x["k"], x["v"], g, beta, state)
        arrays[f"{key}/g"] = g
        arrays[f"{key}/beta"] = beta
        arrays[f"{key}/y"] = y
        arrays[f"{key}/state"] = new_state

    # 4. The whole layer, through the reference's Qwen3_5LinearAttention.
    lin = qc.Qwen3_5LinearAttention(
        num_key_heads=LAYER["hk"], num_value_heads=LAYER["hv"],
        key_head_dim=LAYER["dk"], value_head_dim=LAYER["dv"], conv_kernel_dim=LAYER["kernel"],
    )
    quant = cfg.QuantScheme(bits=4, group_size=64)
    config = qc.Qwen3_5Config(
        num_layers=1, hidden_size=LAYER["hidden"], vocab_size=64, rms_norm_eps=LAYER["eps"],
        num_attention_heads=4, num_key_value_heads=2, head_dim=32, rope_theta=10000.0,
        rotary_dim=8, is_linear_per_layer=(True,), linear=lin, num_experts=4,
        experts_per_token=2, moe_intermediate_size=32, shared_expert_intermediate_size=64,
        norm_topk_prob=True, expert_quant=quant, router_quant=quant,
        shared_gate_quant=quant, other_quant=quant,
    )

    def fresh_cache():
        return rc.RecurrentCache(
            conv_kernel_dim=LAYER["kernel"], conv_dim=lin.conv_dim,
            num_value_heads=LAYER["hv"], value_head_dim=LAYER["dv"], key_head_dim=LAYER["dk"],
        )

    def build(w):
        return la.Qwen3_5LinearAttention(config, **{k: w[k] for k in (
            "in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b", "conv1d_weight",
            "A_log", "dt_bias", "norm_weight", "out_proj")})

    # 4a. One call of 1 and of 6 tokens from a fresh cache (seed 0 / x seed 100).
    for seq_len in (1, 6):
        w, x = layer_case(0, 100, seq_len)
        key = f"layer_fresh_{seq_len}"
        manifest["inputs"][key] = {k: sha(v) for k, v in {**w, "x": x}.items()}
        cache = fresh_cache()
        out = build(w)(x, cache)
        conv_state, ssm_state = cache.state()
        arrays[f"{key}/out"] = out
        arrays[f"{key}/conv_state"] = conv_state
        arrays[f"{key}/ssm_state"] = ssm_state

    # 4b. 5 tokens stepwise from one cache (seed 1 / x seed 101).
    w, x = layer_case(1, 101, 5)
    manifest["inputs"]["layer_steps"] = {k: sha(v) for k, v in {**w, "x": x}.items()}
    layer = build(w)
    batched = layer(x, fresh_cache())
    cache = fresh_cache()
    stepwise = np.stack([layer(x[t], cache) for t in range(x.shape[0])])
    np.testing.assert_allclose(batched, stepwise, rtol=1e-4, atol=1e-5)
    arrays["layer_steps/out"] = stepwise
    arrays["layer_steps/conv_state"] = cache.state()[0]
    arrays["layer_steps/ssm_state"] = cache.state()[1]
    arrays["layer_steps/size"] = np.array(cache.size)

    # 4c. Four calls of 3 tokens into one cache (seed 2 / x seed 102).
    w, _ = layer_case(2, 102, 1)
    rng = np.random.default_rng(102)
    xs = [rng.standard_normal((3, LAYER["hidden"])).astype(np.float32) for _ in range(4)]
    manifest["inputs"]["layer_chunks"] = {k: sha(v) for k, v in {**w, "x": np.stack(xs)}.items()}
    layer = build(w)
    cache = fresh_cache()
    outs = [layer(xc, cache) for xc in xs]
    arrays["layer_chunks/out"] = np.concatenate(outs)
    arrays["layer_chunks/conv_state"] = cache.state()[0]
    arrays["layer_chunks/ssm_state"] = cache.state()[1]
    arrays["layer_chunks/size"] = np.array(cache.size)

    # 5. The softmax-attention layer, through the reference's Qwen3_5Attention
    #    and GrowingKVCache (float32, dense projections).
    at = refmods["attention"]
    kvc = refmods["kv_cache"]
    attn_config = qc.Qwen3_5Config(
        num_layers=1, hidden_size=ATTN["hidden"], vocab_size=64, rms_norm_eps=ATTN["eps"],
        num_attention_heads=ATTN["heads"], num_key_value_heads=ATTN["kv_heads"], head_dim=ATTN["head_dim"],
        rope_theta=ATTN["theta"], rotary_dim=ATTN["rotary"], is_linear_per_layer=(False,), linear=lin,
        num_experts=4, experts_per_token=2, moe_intermediate_size=32, shared_expert_intermediate_size=64,
        norm_topk_prob=True, expert_quant=quant, router_quant=quant, shared_gate_quant=quant, other_quant=quant,
    )

    def attn_layer(w):
        return at.Qwen3_5Attention(attn_config, **w)

    def kv_cache(max_context=16):
        return kvc.GrowingKVCache(max_context=max_context, num_kv_heads=ATTN["kv_heads"],
                                  head_dim=ATTN["head_dim"], dtype=np.float32)

    manifest["source"]["attention"] = "qw/attention.py Qwen3_5Attention + cache/kv_cache.py GrowingKVCache"
    # 5a. One call of 1 and of 6 tokens from a fresh cache (seed 0, x seed 200).
    for seq_len in (1, 6):
        w = attn_case(0)
        x = np.random.default_rng(200).standard_normal((seq_len, ATTN["hidden"])).astype(np.float32)
        key = f"attn_fresh_{seq_len}"
        manifest["inputs"][key] = {k: sha(v) for k, v in {**w, "x": x}.items()}
        cache = kv_cache()
        arrays[f"{key}/out"] = attn_layer(w)(x, cache)
        keys, values = cache.state()
        arrays[f"{key}/keys"], arrays[f"{key}/values"] = keys, values
    # 5b. Five decode steps against one batched call (seed 1, x seed 201).
    w = attn_case(1)
    x = np.random.default_rng(201).standard_normal((5, ATTN["hidden"])).astype(np.float32)
    manifest["inputs"]["attn_steps"] = {k: sha(v) for k, v in {**w, "x": x}.items()}
    layer = attn_layer(w)
    batched = layer(x, kv_cache())
    cache = kv_cache()
    stepwise = np.stack([layer(x[t], cache) for t in range(5)])
    np.testing.assert_allclose(batched, stepwise, rtol=1e-3, atol=1e-4)
    arrays["attn_steps/out"] = stepwise
    arrays["attn_steps/batched"] = batched
    # 5c. Three calls of 4 tokens into one cache: the causal mask of a call
    #     that starts at an offset (seed 3, x seed 203).
    w = attn_case(3)
    xs = np.random.default_rng(203).standard_normal((3, 4, ATTN["hidden"])).astype(np.float32)
    manifest["inputs"]["attn_chunks"] = {k: sha(v) for k, v in {**w, "x": xs}.items()}
    layer = attn_layer(w)
    cache = kv_cache()
    arrays["attn_chunks/out"] = np.concatenate([layer(xc, cache) for xc in xs])
    arrays["attn_chunks/keys"], arrays["attn_chunks/values"] = cache.state()

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden_manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    size = os.path.getsize(os.path.join(HERE, "golden.npz"))
    print(f"wrote {len(arrays)} arrays ({size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
