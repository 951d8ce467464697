"""Benchmark of the gated-delta hot path on B200 (one JSON line on rank 0).

Default workload: config 2, the decode step at the Qwen3.5-MoE linear-attention
shape (B=64 sequences x 1 token, 16 key / 32 value heads, d=128, bf16 q/k/v,
fp32 state [64, 32, 128, 128]), state carried from step to step. A step is
one decode launch over the batch; ``value`` is the state HBM traffic
(algorithmic bytes) per second over all ranks. The same line carries the
prefill number of config 3 (T=8192) under ``"prefill"``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|varlen|prefill|block|qproj|attn|layerdecode] [--tokens M]

``--workload varlen`` is config 5 instead: 64 packed sequences (lengths
``default_rng(1).integers(256, 16384, 64, endpoint=True)``, 516,496 tokens)
split across the ranks by longest-processing-time bin packing, one prefill
over each rank's sequences followed by 256 decode steps; ``value`` is the
prefill rate in tokens/s over all ranks (strong scaling: the total is fixed),
and the decode phase is reported beside it.

``--workload qproj`` times only the 4-bit quantized in-projection (12,352 x
2,048) at ``--tokens`` rows, ``--workload attn`` only the attention core
(prefill of ``--tokens`` tokens, or one decode token against 4,096 cached
positions with ``--tokens 1``), ``--workload layerdecode`` the
linear-attention layer at one decode token launched eagerly, for profiling
those kernels.  The
default line also carries ``"layer"``: config 4 from hidden states in to
hidden states out, with 4-bit affine projections around the fused block.

``--impl reference`` times the reference's CPU path (its ops-path recurrence,
restated on torch's CPU backend with every host thread; MLX is not
installable here) on the same workload, rank 0 only.

Multi-GPU (torchrun, one rank per GPU): each rank decodes its own batch of 64
sequences (sequence sharding, no collective on the data path), timing is the
max over ranks, ``scaling`` is weak. The line's ``"sharded"`` object carries
the strong-scaled configurations at every world size (N=1 included, as the
base of the curve): config 5 LPT-sharded by sequence, and config 3 sharded by
value head with the NCCL all-gather of its outputs timed apart.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-lean-moe_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "GDN prefill tok/s & decode state HBM GB/s (% peak) at 1/2/4/8 B200 vs MLX CPU"
B, HK, HV, D = 64, 16, 32, 128
STATE_BYTES = 2 * B * HV * D * D * 4  # read + write of the fp32 state
DECODE_BYTES = STATE_BYTES + 2 * B * HK * D * 2 + B * HV * D * 2 + 2 * B * HV * 4 + B * HV * D * 4
# DRAM bytes per decode_kernel launch at config 2 (read + write), averaged
# over three consecutive launches of the back-to-back timed loop captured
# with the cache left alone between them (profiles/decode_config2.md).
DECODE_NCU_TRAFFIC = 132_350_464 + 132_196_352
DECODE_NCU_SOURCE = ("ncu --cache-control none capture of launches 11-13 of the back-to-back loop (mean "
                     "dram__bytes_read.sum 132,350,464 + dram__bytes_write.sum 132,196,352 per launch; "
                     "algorithmic 270,548,992)")
PREFILL_T = 8192
PREFILL_FLOP = 182_955 * PREFILL_T * HV  # chunked WY count per token-head: (10 C^2 d + 6 C d^2 + 2/3 C^3) / C, C = 64, d = 128
# Algorithmic bytes of one config-3 call: q, k (bf16) + v (bf16) + g, beta (fp32) + y (fp32) + final state (fp32).
PREFILL_BYTES = 2 * PREFILL_T * HK * D * 2 + PREFILL_T * HV * D * 2 + 2 * PREFILL_T * HV * 4 + PREFILL_T * HV * D * 4 \
    + HV * D * D * 4
# Counters of the config-3 prefill kernels from one ncu capture of a call
# (profiles/chunked_prefill_config3.md): the tensor pipe's share of the scan
# kernels' active cycles, and the DRAM bytes of all the call's kernels.
PREFILL_NCU = {"tensor_pipe_frac": 0.296, "traffic": 581_989_376,
               "ncu_source": "ncu --set full capture of one config-3 call (chunk_prep x2, chunk_scan x2, "
                             "state_combine; profiles/chunked_prefill_config3.md): tensor_pipe_frac = "
                             "sm__pipe_tensor_cycles_active of the scan launches (30.1 % and 29.2 % of their "
                             "SMs' active cycles, time-weighted); traffic = dram__bytes_read.sum + "
                             "dram__bytes_write.sum of the five launches"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def bf16_round(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def decode_step_inputs(seed):
    """Config 2 per-step draws (q, k L2-normalised, v ~ N(0,1), beta =
    sigmoid(N), g = -softplus(N)), q/k/v as bf16."""
    rng = np.random.default_rng(seed)
    l2n = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = torch.from_numpy(l2n(rng.standard_normal((B, HK, D), dtype=np.float32))).to(torch.bfloat16)
    k = torch.from_numpy(l2n(rng.standard_normal((B, HK, D), dtype=np.float32))).to(torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((B, HV, D), dtype=np.float32)).to(torch.bfloat16)
    beta = torch.from_numpy(1 / (1 + np.exp(-rng.standard_normal((B, HV), dtype=np.float32))))
    g = torch.from_numpy(-np.logaddexp(np.float32(0), rng.standard_normal((B, HV), dtype=np.float32)))
    return q, k, v, g.float(), beta.float()


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.proc = None
        self.bus = None
        try:
            props = torch.cuda.get_device_properties(device_index)
            dom, bus, dev = (getattr(props, f"pci_{x}_id", None) for x in ("domain", "bus", "device"))
            if all(isinstance(x, int) for x in (dom, bus, dev)):
                self.bus = f"{dom:08x}:{bus:02x}:{dev:02x}.0"
        except Exception:
            pass
        self.local = device_index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is None:
            return
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            self.rows.append(parts)

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        mine = [r for r in rows if self.bus and r[1].lower().endswith(self.bus[-12:])] or \
               [r for r in rows if r[0] == str(self.local)] or rows
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in mine for i, x in enumerate(r[6:10]) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(mine[0][3]) if mine[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(mine)}


def clocks_under_load(fn, device, seconds=1.2):
    """Clocks while fn() runs back to back for about `seconds` (outside any
    timed region): the SM clock the chunked kernels actually get under load."""
    with ClockSampler(device.index or 0) as sampler:
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end:
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
    return sampler.summary()


def cpu_decode_sample(budget_s=10.0):
    """The reference's CPU path for config 2: per sequence, the ops-path
    recurrence for one token (torch CPU, all threads). Runs whole steps over
    all 64 sequences until ~budget_s has passed (at least one)."""
    from oracle.gdn_torch_cpu import gated_delta_scan_ops

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    state = torch.from_numpy((rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02))
    steps, t0 = 0, time.perf_counter()
    while True:
        q, k, v, g_log, beta = decode_step_inputs(100 + steps)
        q, k, v = q.float(), k.float(), v.float()
        g = torch.exp(g_log)
        for b in range(B):
            _, state[b] = gated_delta_scan_ops(q[b : b + 1], k[b : b + 1], v[b : b + 1], g[b : b + 1],
                                               beta[b : b + 1], state[b])
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= budget_s:
            break
    return steps, elapsed


def mlx_probe():
    """Whether the reference's own CPU path could run on this host: it needs
    mlx (``import mlx.core``, mlx 0.32.2 in the reference's lock file) and
    the reference's sources. Returns a one-line finding for the JSON line."""
    try:
        import mlx.core as mx  # noqa: F401
    except Exception as e:  # ImportError on hosts without mlx
        return f"import mlx.core failed ({type(e).__name__}: {e}); the torch-CPU restatement is timed instead"
    return ("import mlx.core succeeded, but the reference's sources are not on this host; the torch-CPU "
            "restatement is timed instead")


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args, world, rank):
    """``--impl reference``: the reference's CPU path on the same workload,
    rank 0 only (other ranks exit without work)."""
    if rank == 0 and args.workload == "varlen":
        cores = os.cpu_count() or 1
        rates = [cpu_prefill_sample() for _ in range(args.warmup + args.steps)][args.warmup:]
        value = statistics.mean(rates)
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 512 / value * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config 5)",
            "config": {"workload": "config 5 prefill, sampled: 512 tokens of one sequence per step",
                       "global_batch": 1, "seq_len": 512, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": "512 tokens of one config-5 sequence per step (torch-CPU restatement of the "
                                       "reference's ops path); MLX probe: " + mlx_probe()},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return
    if rank == 0:
        cores = os.cpu_count() or 1
        torch.set_num_threads(cores)
        from oracle.gdn_torch_cpu import gated_delta_scan_ops

        rng = np.random.default_rng(0)
        state = torch.from_numpy(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02)
        times = []
        for step in range(args.warmup + args.steps):
            q, k, v, g_log, beta = decode_step_inputs(100 + step)
            q, k, v = q.float(), k.float(), v.float()
            g = torch.exp(g_log)
            t0 = time.perf_counter()
            for b in range(B):
                _, state[b] = gated_delta_scan_ops(q[b : b + 1], k[b : b + 1], v[b : b + 1], g[b : b + 1],
                                                   beta[b : b + 1], state[b])
            if step >= args.warmup:
                times.append(time.perf_counter() - t0)
        total = sum(times)
        value = DECODE_BYTES * len(times) / total / 1e9
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config 2 distributions)",
            "config": {"workload": "decode, config 2: B=64 x 1 token, 16/32 heads, d=128, fp32 state, "
                                   "state carried", "global_batch": B, "seq_len": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} full decode steps of 64 sequences (torch-CPU restatement "
                                       "of the reference's ops path); MLX probe: " + mlx_probe()},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)


def measure_prefill(device, iters=3, warmup=2, clocks=False):
    """Config 3: one sequence of 8192 tokens, bf16 q/k/v, fp32 state from 0.
    Median device time of one call (ms); with clocks=True also the clocks
    of the same call run back to back for about a second."""
    import gdn_b200

    rng = np.random.default_rng(3)
    l2n = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = torch.from_numpy(l2n(rng.standard_normal((PREFILL_T, HK, D), dtype=np.float32))).to(device, torch.bfloat16)
    k = torch.from_numpy(l2n(rng.standard_normal((PREFILL_T, HK, D), dtype=np.float32))).to(device, torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((PREFILL_T, HV, D), dtype=np.float32)).to(device, torch.bfloat16)
    beta = torch.sigmoid(torch.randn(PREFILL_T, HV, device=device, generator=torch.Generator(device).manual_seed(1)))
    g = -torch.nn.functional.softplus(torch.randn(PREFILL_T, HV, device=device,
                                                  generator=torch.Generator(device).manual_seed(2)))
    state = torch.zeros(1, HV, D, D, device=device)
    out = torch.empty(PREFILL_T, HV, D, device=device)
    st_out = torch.empty_like(state)
    for _ in range(warmup):
        gdn_b200.gated_delta_scan_varlen(q, k, v, g, beta, state, g_is_log=True, state_out=st_out, out=out)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * iters)]
    for i in range(iters):
        ev[2 * i].record()
        gdn_b200.gated_delta_scan_varlen(q, k, v, g, beta, state, g_is_log=True, state_out=st_out, out=out)
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(iters))
    if clocks:
        return ms, clocks_under_load(lambda: gdn_b200.gated_delta_scan_varlen(
            q, k, v, g, beta, state, g_is_log=True, state_out=st_out, out=out), device)
    return ms


def measure_block(device, iters=3, clocks=False):
    """Config 4: the fused block, B=8 x T=4096, bf16 mixed projection.
    Returns (ms, tokens), and with clocks=True the clocks of the call run
    back to back for about a second."""
    import gdn_b200
    from gdn_b200.linear_attention import LinearAttentionShape

    shape = LinearAttentionShape(HK, HV, D, D, 4)
    Bb, T = 8, 4096
    gen = torch.Generator(device).manual_seed(4)
    mixed = torch.randn(Bb * T, shape.mixed_width, device=device, generator=gen).bfloat16()
    conv_w = torch.randn(shape.conv_dim, 4, device=device, generator=gen) * 0.1
    A_log = torch.rand(HV, device=device, generator=gen) * 1.5
    dt_bias = torch.randn(HV, device=device, generator=gen) * 0.1
    norm_w = torch.ones(D, device=device)
    conv_state = torch.zeros(Bb, 3, shape.conv_dim, device=device)
    ssm = torch.zeros(Bb, HV, D, D, device=device)
    out = torch.empty(Bb * T, HV, D, device=device, dtype=torch.bfloat16)

    def run():
        conv_state.zero_()
        ssm.zero_()
        gdn_b200.gated_delta_block(mixed, shape, conv_w, A_log, dt_bias, norm_w, 1e-6, conv_state, ssm,
                                   n_seqs=Bb, out=out)

    for _ in range(2):
        run()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * iters)]
    for i in range(iters):
        ev[2 * i].record()
        run()
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(iters))
    if clocks:
        return ms, Bb * T, clocks_under_load(run, device)
    return ms, Bb * T


HIDDEN = 2048


def quantized_weights(device, rows, cols, gen, bits=4, group=64):
    """Random affine-quantized weights in the reference's storage (uint32 words
    as int32, bf16 scales and biases); values of a trained layer's scale."""
    words = torch.randint(-2**31, 2**31 - 1, (rows, cols * bits // 32), dtype=torch.int32, device=device,
                          generator=gen)
    scales = (torch.rand(rows, cols // group, device=device, generator=gen) * 2e-3 + 1e-3).bfloat16()
    biases = (-(2 ** (bits - 1)) * scales.float()).bfloat16()
    return {"weight": words, "scales": scales, "biases": biases}


def measure_layer(device, iters=3):
    """Config 4 as a whole layer: hidden states in (B=8 x T=4096, 2048 wide,
    bf16), the four input projections as one 4-bit quantized GEMM into the
    mixed row, the fused block, the 4-bit out_proj, hidden states out."""
    import gdn_b200
    from gdn_b200 import LinearWeights, QuantScheme, concat_rows, quantized_linear
    from gdn_b200.linear_attention import LinearAttentionShape

    shape = LinearAttentionShape(HK, HV, D, D, 4)
    Bb, T = 8, 4096
    q4 = QuantScheme(bits=4, group_size=64)
    gen = torch.Generator(device).manual_seed(5)
    in_proj = concat_rows([LinearWeights(quantized_weights(device, r, HIDDEN, gen), q4)
                           for r in (shape.conv_dim, shape.value_dim, HV, HV)])
    out_proj = LinearWeights(quantized_weights(device, HIDDEN, shape.value_dim, gen), q4)
    x = torch.randn(Bb * T, HIDDEN, device=device, generator=gen).bfloat16()
    conv_w = torch.randn(shape.conv_dim, 4, device=device, generator=gen) * 0.1
    A_log = torch.rand(HV, device=device, generator=gen) * 1.5
    dt_bias = torch.randn(HV, device=device, generator=gen) * 0.1
    norm_w = torch.ones(D, device=device)
    conv_state = torch.zeros(Bb, 3, shape.conv_dim, device=device)
    ssm = torch.zeros(Bb, HV, D, D, device=device)
    core = torch.empty(Bb * T, HV, D, device=device, dtype=torch.bfloat16)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def run(record):
        conv_state.zero_()
        ssm.zero_()
        if record:
            ev[0].record()
        mixed = quantized_linear(x, in_proj)
        if record:
            ev[1].record()
        gdn_b200.gated_delta_block(mixed, shape, conv_w, A_log, dt_bias, norm_w, 1e-6, conv_state, ssm,
                                   n_seqs=Bb, out=core)
        if record:
            ev[2].record()
        out = quantized_linear(core.view(Bb * T, -1), out_proj)
        if record:
            ev[3].record()
        return out

    for _ in range(2):
        run(False)
    torch.cuda.synchronize()
    parts = []
    for _ in range(iters):
        run(True)
        torch.cuda.synchronize()
        parts.append([ev[i].elapsed_time(ev[i + 1]) for i in range(3)])
    med = [statistics.median(p[i] for p in parts) for i in range(3)]
    n_tok = Bb * T
    gemm_flop = 2 * n_tok * HIDDEN * (shape.mixed_width + shape.value_dim)
    return {"tokens": n_tok, "in_proj_ms": med[0], "block_ms": med[1], "out_proj_ms": med[2],
            "ms": sum(med), "gemm_flop": gemm_flop}


def linear_layer_at_decode(device):
    """Qwen3_5LinearAttention at the model's shape (16/32 heads of 128,
    hidden 2,048, 4-bit group-64 projections), its RecurrentCache and one
    decode token of hidden state."""
    import gdn_b200
    from gdn_b200 import LinearWeights, QuantScheme
    from gdn_b200.linear_attention import LinearAttentionShape

    shape = LinearAttentionShape(HK, HV, D, D, 4)
    q4 = QuantScheme(bits=4, group_size=64)
    gen = torch.Generator(device).manual_seed(8)
    qw = lambda rows, cols: LinearWeights(quantized_weights(device, rows, cols, gen), q4)
    layer = gdn_b200.Qwen3_5LinearAttention(
        shape, 1e-6, qw(shape.conv_dim, HIDDEN), qw(shape.value_dim, HIDDEN), qw(HV, HIDDEN), qw(HV, HIDDEN),
        torch.randn(shape.conv_dim, 4, 1, device=device, generator=gen) * 0.1,
        torch.rand(HV, device=device, generator=gen) * 1.5, torch.randn(HV, device=device, generator=gen) * 0.1,
        torch.ones(D, device=device), qw(HIDDEN, shape.value_dim))
    cache = gdn_b200.RecurrentCache(4, shape.conv_dim, HV, D, D, device=device)
    x1 = torch.randn(HIDDEN, device=device, generator=gen).bfloat16()
    return layer, cache, x1


def measure_layer_decode(device, iters=3):
    """The linear-attention layer at one decode token, as a CUDA-graph
    replay: the fused in-projection GEMV, the fused block on one token, the
    out_proj GEMV."""
    layer, cache, x1 = linear_layer_at_decode(device)
    layer(x1, cache)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            for _ in range(20):
                layer(x1, cache)
    torch.cuda.synchronize()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = []
    for _ in range(iters):
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1) / 20)
    del graph
    return statistics.median(ms) * 1e3


def measure_attention(device, iters=3):
    """The softmax-attention core at the model's attention shape (16 query
    heads over 2 key/value heads of 256, rotary 64, bf16): a 4,096-token
    prefill from an empty cache, and one decode token against 4,096 cached
    positions."""
    import gdn_b200
    from gdn_b200 import AttentionShape, GrowingKVCache

    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    L = 4096
    gen = torch.Generator(device).manual_seed(7)
    qg = torch.randn(L, 16 * 512, device=device, generator=gen).bfloat16()
    k = torch.randn(L, 2 * 256, device=device, generator=gen).bfloat16()
    v = torch.randn(L, 2 * 256, device=device, generator=gen).bfloat16()
    qn = torch.ones(256, device=device)

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ms = []
        for _ in range(iters):
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
        return statistics.median(ms)

    def prefill():
        cache = GrowingKVCache(L + 1, 2, 256, dtype=torch.bfloat16, device=device)
        cache.reserve(L)
        gdn_b200.attention_core(qg, k, v, qn, qn, shape, 1e-6, cache)

    pre_ms = timed(prefill)
    cache = GrowingKVCache(L + 64, 2, 256, dtype=torch.bfloat16, device=device)
    gdn_b200.attention_core(qg, k, v, qn, qn, shape, 1e-6, cache)

    # decode as a CUDA-graph replay (device time; the Python call alone costs
    # more than the three launches): the same position every time, 4,096
    # cached keys and values.  Thread-local capture: under torchrun the
    # process-group watchdog thread queries events while this thread captures.
    cache.commit(L)
    gdn_b200.attention_core(qg[:1], k[:1], v[:1], qn, qn, shape, 1e-6, cache)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        cache.commit(L)
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            for _ in range(20):
                gdn_b200.attention_core(qg[:1], k[:1], v[:1], qn, qn, shape, 1e-6, cache)
                cache.commit(L)
    torch.cuda.synchronize()
    dec_ms = timed(graph.replay) / 20
    del graph

    # the whole layer at one decode token: the fused 4-bit q|gate|k|v GEMV,
    # the core, the 4-bit o_proj GEMV (hidden 2,048, group 64)
    from gdn_b200 import LinearWeights, QuantScheme, Qwen3_5Attention

    q4 = QuantScheme(bits=4, group_size=64)
    qw = lambda rows, cols: LinearWeights(quantized_weights(device, rows, cols, gen), q4)
    layer = Qwen3_5Attention(shape, 1e-6, qw(16 * 512, HIDDEN), qn, qw(2 * 256, HIDDEN), qn, qw(2 * 256, HIDDEN),
                             qw(HIDDEN, 16 * 256))
    x1 = torch.randn(HIDDEN, device=device, generator=gen).bfloat16()
    cache.commit(L)
    layer(x1, cache)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        cache.commit(L)
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            for _ in range(20):
                layer(x1, cache)
                cache.commit(L)
    torch.cuda.synchronize()
    layer_ms = timed(graph.replay) / 20
    del graph
    flop = 4 * 256 * 16 * L * (L + 1) / 2
    kv_bytes = 2 * 2 * (L + 1) * 256 * 2
    return {"prefill_ms": pre_ms, "prefill_tflops": flop / (pre_ms / 1e3) / 1e12,
            "decode_us": dec_ms * 1e3, "decode_kv_gbs": kv_bytes / (dec_ms / 1e3) / 1e9,
            "layer_decode_us": layer_ms * 1e3}


def run_attn(args):
    """Only the softmax-attention core at the model's attention shape (16
    query heads over 2 key/value heads of 256, rotary 64, bf16): with
    ``--tokens`` L > 1 a prefill of L tokens from an empty cache per step,
    with L = 1 one decode token against 4,096 cached positions per step; for
    profiling the attention kernels on their own."""
    import gdn_b200
    from gdn_b200 import AttentionShape, GrowingKVCache

    device = torch.device("cuda", 0)
    shape = AttentionShape(16, 2, 256, 64, 10000000.0)
    L = max(args.tokens, 4096)
    gen = torch.Generator(device).manual_seed(7)
    qg = torch.randn(L, 16 * 512, device=device, generator=gen).bfloat16()
    k = torch.randn(L, 2 * 256, device=device, generator=gen).bfloat16()
    v = torch.randn(L, 2 * 256, device=device, generator=gen).bfloat16()
    qn = torch.ones(256, device=device)
    cache = GrowingKVCache(L + 64, 2, 256, dtype=torch.bfloat16, device=device)
    n = args.tokens
    if n == 1:
        gdn_b200.attention_core(qg[:4096], k[:4096], v[:4096], qn, qn, shape, 1e-6, cache)

    def step():
        cache.commit(4096 if n == 1 else 0)
        gdn_b200.attention_core(qg[:n], k[:n], v[:n], qn, qn, shape, 1e-6, cache)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    flop = 4 * 256 * 16 * (n * 4096 if n == 1 else n * (n + 1) / 2)
    print(json.dumps({"metric": "attention core TFLOP/s", "value": flop / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "config": {"workload": (f"prefill {n} tokens" if n > 1 else "decode, 4,096 cached") +
                                 ", 16/2 heads of 256, rotary 64, bf16"},
                      "dtype": "bf16", "data": "synthetic"}), flush=True)


def run_prefill(args):
    """Only config 3 (one sequence of 8,192 tokens, 16/32 heads of 128, bf16
    q/k/v, fp32 state from 0), K calls back to back; for profiling the
    prefill kernels on their own."""
    device = torch.device("cuda", 0)
    ms, clk = measure_prefill(device, iters=max(args.steps, 1), warmup=args.warmup, clocks=True)
    _, tc_peak, _ = peaks()
    print(json.dumps({"metric": "config-3 prefill tok/s", "value": PREFILL_T / (ms / 1e3), "unit": "tok/s",
                      "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "achieved_tflops": PREFILL_FLOP / (ms / 1e3) / 1e12,
                      "frac_of_bf16_peak": PREFILL_FLOP / (ms / 1e3) / 1e12 / tc_peak,
                      "config": {"workload": "config 3: B=1, T=8192, 16/32 heads, d=128, bf16 q/k/v, fp32 out"},
                      "clocks_under_load": clk, "dtype": "bf16", "data": "synthetic"}), flush=True)


def run_block(args):
    """Only config 4 (the fused block over B=8 x T=4096, bf16 mixed
    projection), K calls; for profiling the block's kernels on their own."""
    device = torch.device("cuda", 0)
    ms, tok, clk = measure_block(device, iters=max(args.steps, 1), clocks=True)
    _, tc_peak, _ = peaks()
    flop = (PREFILL_FLOP // PREFILL_T) * tok
    print(json.dumps({"metric": "config-4 fused block tok/s", "value": tok / (ms / 1e3), "unit": "tok/s",
                      "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "achieved_tflops": flop / (ms / 1e3) / 1e12, "frac_of_bf16_peak": flop / (ms / 1e3) / 1e12 / tc_peak,
                      "config": {"workload": "config 4: fused block, B=8 x T=4096, 16/32 heads, d=128"},
                      "clocks_under_load": clk, "dtype": "bf16", "data": "synthetic"}), flush=True)


def run_layerdecode(args):
    """Only the linear-attention layer at one decode token, launched eagerly
    (one kernel after another, as ncu lists them); for profiling the decode
    chain's kernels."""
    device = torch.device("cuda", 0)
    layer, cache, x1 = linear_layer_at_decode(device)
    for _ in range(args.warmup):
        layer(x1, cache)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        layer(x1, cache)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    print(json.dumps({"metric": "linear-attention layer decode step", "value": ms * 1e3, "unit": "us",
                      "higher_is_better": False, "steps": args.steps, "warmup": args.warmup,
                      "config": {"workload": "Qwen3_5LinearAttention at one decode token, 16/32 heads of 128, "
                                             "hidden 2,048, 4-bit projections, launched eagerly"},
                      "dtype": "bf16", "data": "synthetic"}), flush=True)


def run_qproj(args):
    """Only the quantized in-projection (12,352 x 2,048, 4-bit, group 64) at
    ``--tokens`` rows: the GEMV up to 16 tokens, the tiled GEMM beyond; for
    profiling the projection kernels on their own."""
    from gdn_b200 import QuantScheme, quantized_linear

    device = torch.device("cuda", 0)
    gen = torch.Generator(device).manual_seed(6)
    n = 2 * HK * D + 2 * HV * D + 2 * HV  # q|k|v|z|b|a: 12,352
    w = quantized_weights(device, n, HIDDEN, gen)
    q4 = QuantScheme(bits=4, group_size=64)
    x = torch.randn(args.tokens, HIDDEN, device=device, generator=gen).bfloat16()
    for _ in range(args.warmup):
        quantized_linear(x, w, q4)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        quantized_linear(x, w, q4)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    flop = 2 * args.tokens * n * HIDDEN
    print(json.dumps({"metric": "quantized in-projection TFLOP/s", "value": flop / (ms / 1e3) / 1e12,
                      "unit": "TFLOP/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "config": {"workload": f"in_proj {args.tokens} x {n} x {HIDDEN}, 4-bit affine, group 64"},
                      "dtype": "bf16", "data": "synthetic"}), flush=True)


def cpu_prefill_sample(n_tokens=512):
    """The reference's CPU path on the first ``n_tokens`` tokens of config 5's
    first sequence (all host threads); returns tokens/s."""
    from oracle.gdn_torch_cpu import gated_delta_scan_ops

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(5)
    q = torch.nn.functional.normalize(torch.randn(n_tokens, HK, D, generator=g), dim=-1).bfloat16().float()
    k = torch.nn.functional.normalize(torch.randn(n_tokens, HK, D, generator=g), dim=-1).bfloat16().float()
    v = torch.randn(n_tokens, HV, D, generator=g).bfloat16().float()
    beta = torch.sigmoid(torch.randn(n_tokens, HV, generator=g))
    gm = torch.exp(-torch.nn.functional.softplus(torch.randn(n_tokens, HV, generator=g)))
    s0 = torch.randn(HV, D, D, generator=g) * 0.02
    t0 = time.perf_counter()
    gated_delta_scan_ops(q, k, v, gm, beta, s0)
    return n_tokens / (time.perf_counter() - t0)


def varlen_setup(world, rank, device):
    """Config 5 on this rank's share of the 64 sequences (LPT partition of
    the lengths): the packed inputs, one prefill over them and 256 decode
    steps with the carried states. Returns (prefill, decode, info)."""
    import gdn_b200
    from gdn_b200.sharding import lpt_partition

    lengths = np.random.default_rng(1).integers(256, 16384, size=64, endpoint=True)
    parts = lpt_partition(lengths, world)
    mine = parts[rank]
    my_len = [int(lengths[i]) for i in mine]
    n_loc = len(my_len)
    n_tok = int(sum(my_len))
    gen = torch.Generator(device).manual_seed(100 + rank)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(my_len)]), dtype=torch.int64, device=device)
    q = torch.nn.functional.normalize(torch.randn(n_tok, HK, D, device=device, generator=gen), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(n_tok, HK, D, device=device, generator=gen), dim=-1).bfloat16()
    v = torch.randn(n_tok, HV, D, device=device, generator=gen).bfloat16()
    beta = torch.sigmoid(torch.randn(n_tok, HV, device=device, generator=gen))
    g_log = -torch.nn.functional.softplus(torch.randn(n_tok, HV, device=device, generator=gen))
    s_init = torch.randn(max(n_loc, 1), HV, D, D, device=device, generator=gen) * 0.02
    state = torch.empty_like(s_init)
    out = torch.empty(n_tok, HV, D, device=device)
    dq = torch.nn.functional.normalize(torch.randn(4, max(n_loc, 1), HK, D, device=device, generator=gen), dim=-1).bfloat16()
    dk = torch.nn.functional.normalize(torch.randn(4, max(n_loc, 1), HK, D, device=device, generator=gen), dim=-1).bfloat16()
    dv = torch.randn(4, max(n_loc, 1), HV, D, device=device, generator=gen).bfloat16()
    db = torch.sigmoid(torch.randn(4, max(n_loc, 1), HV, device=device, generator=gen))
    dg = -torch.nn.functional.softplus(torch.randn(4, max(n_loc, 1), HV, device=device, generator=gen))
    dout = torch.empty(max(n_loc, 1), HV, D, device=device)
    n_decode = 256

    def prefill():
        state.copy_(s_init)
        if n_loc:
            gdn_b200.gated_delta_scan_varlen(q, k, v, g_log, beta, state, cu, g_is_log=True, state_out=state,
                                             out=out)

    def decode():
        for i in range(n_decode):
            if n_loc:
                gdn_b200.gated_delta_decode(dq[i % 4, :n_loc], dk[i % 4, :n_loc], dv[i % 4, :n_loc],
                                            dg[i % 4, :n_loc], db[i % 4, :n_loc], state[:n_loc], g_is_log=True,
                                            out=dout[:n_loc])

    loads = [int(sum(int(lengths[i]) for i in p_)) for p_ in parts]
    info = {"lengths": lengths, "n_decode": n_decode, "tokens": int(lengths.sum()),
            "lpt_max_over_mean": max(loads) / (sum(loads) / len(loads))}
    return prefill, decode, info


def time_varlen(prefill, decode, steps, warmup, world, device, sampler=None):
    """Device time (ms, summed over steps, max over ranks) of the config-5
    prefill and of its decode phase."""
    for _ in range(warmup):
        prefill()
        decode()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    pf_ms, dec_ms = 0.0, 0.0
    import contextlib

    with sampler if sampler is not None else contextlib.nullcontext():
        for _ in range(steps):
            ev[0].record()
            prefill()
            ev[1].record()
            decode()
            ev[2].record()
            torch.cuda.synchronize()
            pf_ms += ev[0].elapsed_time(ev[1])
            dec_ms += ev[1].elapsed_time(ev[2])
    if world > 1:
        t = torch.tensor([pf_ms, dec_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        pf_ms, dec_ms = float(t[0]), float(t[1])
        torch.distributed.barrier()
    return pf_ms, dec_ms


def run_varlen(args, world, rank, local):
    """Config 5 on this rank's share of the sequences (see module docstring)."""
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    prefill, decode, info = varlen_setup(world, rank, device)
    sampler = ClockSampler(local)
    pf_ms, dec_ms = time_varlen(prefill, decode, args.steps, args.warmup, world, device, sampler)
    total_tok = info["tokens"]
    n_decode = info["n_decode"]
    dec_bytes = n_decode * (2 * 64 * HV * D * D * 4)  # state read + write of all 64 sequences per step
    hbm_peak, tc_peak, peak_kind = peaks()
    pf_s = pf_ms / 1e3 / args.steps
    line = {
        "metric": METRIC, "value": total_tok / pf_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": (pf_ms + dec_ms) / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 state / bf16 q,k,v",
        "data": "synthetic (seeded; config 5 lengths and value distributions)",
        "config": {"workload": "config 5: 64 packed sequences, 516,496 tokens, LPT-sharded by sequence; prefill "
                               "then 256 decode steps per sequence, no cross-GPU exchange",
                   "global_batch": 64, "seq_len": "256..16384 (packed)", "parallelism": f"sequence-sharded x{world}",
                   "l2": "inputs (4.2 GB of q/k/v) far larger than L2"},
        "prefill": {"ms": pf_ms / args.steps, "achieved_tflops": PREFILL_FLOP / PREFILL_T * total_tok / pf_s / 1e12,
                    "frac_of_bf16_peak": PREFILL_FLOP / PREFILL_T * total_tok / pf_s / 1e12 / (tc_peak * world),
                    "lpt_max_over_mean": info["lpt_max_over_mean"]},
        "decode": {"value": dec_bytes / (dec_ms / 1e3 / args.steps) / 1e9, "unit": "GB/s", "steps": n_decode,
                   "ms": dec_ms / args.steps, "peak": hbm_peak, "peak_kind": peak_kind},
        "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = {"value": cpu_prefill_sample(), "unit": "tok/s", "cores": os.cpu_count() or 1,
                                "kind": "port", "sample": "first 512 tokens of one config-5-shaped sequence "
                                "(torch-CPU restatement of the reference's ops path, all threads); MLX probe: "
                                + mlx_probe()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def measure_sharded(world, rank, device, steps=3):
    """The sharded configurations at this world size (every rank takes part,
    collectives in the same order on all ranks): config 5 LPT-sharded by
    sequence (strong scaling, no collective), and config 3 sharded by value
    head (whole GQA groups) with the NCCL all-gather of the outputs timed
    apart. Device times are max over ranks."""
    import gdn_b200
    from gdn_b200.sharding import all_gather_heads, head_shard

    hbm_peak, tc_peak, _ = peaks()
    res = {}
    prefill, decode, info = varlen_setup(world, rank, device)
    pf_ms, dec_ms = time_varlen(prefill, decode, steps, 1, world, device)
    del prefill, decode
    pf_s = pf_ms / 1e3 / steps
    tflops = PREFILL_FLOP / PREFILL_T * info["tokens"] / pf_s / 1e12
    res["config5"] = {
        "prefill_tok_s": info["tokens"] / pf_s, "prefill_ms": pf_ms / steps, "prefill_tflops": tflops,
        "prefill_frac_of_bf16_peak": tflops / (tc_peak * world), "lpt_max_over_mean": info["lpt_max_over_mean"],
        "decode_gbs": info["n_decode"] * (2 * 64 * HV * D * D * 4) / (dec_ms / 1e3 / steps) / 1e9,
        "decode_ms": dec_ms / steps, "scaling": "strong",
        "note": "64 sequences (516,496 tokens) LPT-packed over the ranks, prefill then 256 decode steps per "
                "sequence; no collective"}
    torch.cuda.empty_cache()

    # config 3 by value head: this rank's GQA groups, then the all-gather
    ks, vs = head_shard(HK, HV, rank, world)
    gen = torch.Generator(device).manual_seed(3)
    q = torch.nn.functional.normalize(torch.randn(PREFILL_T, HK, D, device=device, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(PREFILL_T, HK, D, device=device, generator=gen), dim=-1)
    v = torch.randn(PREFILL_T, HV, D, device=device, generator=gen)
    beta = torch.sigmoid(torch.randn(PREFILL_T, HV, device=device, generator=gen))
    g = -torch.nn.functional.softplus(torch.randn(PREFILL_T, HV, device=device, generator=gen))
    ql, kl, vl = (x.bfloat16().contiguous() for x in (q[:, ks], k[:, ks], v[:, vs]))
    gl, bl = g[:, vs].contiguous(), beta[:, vs].contiguous()
    out = torch.empty(PREFILL_T, HV // world, D, device=device, dtype=torch.bfloat16)

    def scan():
        gdn_b200.gated_delta_scan_varlen(ql, kl, vl, gl, bl, None, g_is_log=True, out=out)

    def gather():
        return all_gather_heads(out, world) if world > 1 else out

    for _ in range(2):
        scan()
        gather()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    scan_ms = ag_ms = 0.0
    for _ in range(steps):
        ev[0].record()
        scan()
        ev[1].record()
        gather()
        ev[2].record()
        torch.cuda.synchronize()
        scan_ms += ev[0].elapsed_time(ev[1])
        ag_ms += ev[1].elapsed_time(ev[2])
    if world > 1:
        t = torch.tensor([scan_ms, ag_ms, scan_ms + ag_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        scan_ms, ag_ms, tot_ms = (float(x) for x in t)
        torch.distributed.barrier()
    else:
        tot_ms = scan_ms + ag_ms
    res["config3_head_sharded"] = {
        "tok_s": PREFILL_T / (tot_ms / 1e3 / steps), "ms": tot_ms / steps, "scan_ms": scan_ms / steps,
        "all_gather_ms": ag_ms / steps, "heads_per_rank": HV // world, "scaling": "strong",
        "note": "T=8192, value heads split over the ranks with their key heads, bf16 outputs all-gathered "
                "(NCCL all_gather_into_tensor) into [8192, 32, 128] on every rank"}

    if world > 1:
        # the same, with the gather fused into the scan: each rank's output
        # tiles go to every rank's [8192, 32, 128] buffer over NVLink from the
        # scan kernel (gdn_scan_gathered), then a one-element all-reduce
        from gdn_b200.sharding import GatheredHeads

        gh = GatheredHeads(PREFILL_T, HV, D, torch.bfloat16, device)
        for _ in range(2):
            gh.scan(ql, kl, vl, gl, bl, None, vs.start, g_is_log=True)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            gh.scan(ql, kl, vl, gl, bl, None, vs.start, g_is_log=True)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        fused_ms = float(t.item()) / steps
        gh.close()
        res["config3_head_sharded_fused_gather"] = {
            "tok_s": PREFILL_T / (fused_ms / 1e3), "ms": fused_ms, "heads_per_rank": HV // world,
            "scaling": "strong", "kernel": "chunk_scan_kernel with peer stores (gdn_scan_gathered)",
            "note": "as config3_head_sharded, but the scan's output stage writes each bf16 output tile into every "
                    "rank's [8192, 32, 128] buffer (16-byte stores over NVLink to CUDA-IPC mappings), then a "
                    "one-element NCCL all-reduce orders the readers; no all-gather"}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode only: no e2e, prefill or CPU legs (for profiler runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg (profiler runs)")
    ap.add_argument("--workload", choices=["decode", "varlen", "prefill", "block", "qproj", "attn", "layerdecode"],
                    default="decode")
    ap.add_argument("--tokens", type=int, default=4096, help="rows of x for --workload qproj / attn")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload in ("qproj", "attn", "layerdecode", "prefill", "block"):
        if args.impl == "reference":
            why = ("a profiling workload of this build's own kernels; the reference arm times config 2 (default) "
                   "and config 5 (--workload varlen)") if args.workload in ("prefill", "block") else (
                   "the reference's quantized matmul and attention are MLX's (mx.quantized_matmul, "
                   "mx.fast.scaled_dot_product_attention), not installable on this box")
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
            return
        return {"qproj": run_qproj, "attn": run_attn, "layerdecode": run_layerdecode,
                "prefill": run_prefill, "block": run_block}[args.workload](args)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if args.workload == "varlen":
        return run_varlen(args, world, rank, local)

    import gdn_b200

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    hbm_peak, tc_peak, peak_kind = peaks()

    # --- device-resident decode (value) --------------------------------
    rng = np.random.default_rng(1000 + rank)
    state = torch.from_numpy(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02).to(device)
    n_inputs = 8
    dev_inputs = [tuple(x.to(device) for x in decode_step_inputs(rank * 1000 + i)) for i in range(n_inputs)]
    out = torch.empty(B, HV, D, device=device)
    # L2 flush between timed steps: write 256 MiB (> 126 MB L2), then read a
    # second 256 MiB buffer so no dirty lines of the flush are left to be
    # written back during the timed kernel.
    flush_w = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    flush_r = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=device)

    # The timed loop calls the C ABI directly with argument blocks built once
    # (gdn_decode, in place on `state`), so host-side Python cannot leave the
    # GPU idle inside a timed step.
    import ctypes

    from gdn_b200 import _lib
    from gdn_b200.gated_delta import _scan_args

    lib = _lib.load()
    stream_handle = torch.cuda.current_stream(device).cuda_stream
    decode_args = []
    for q, k, v, g, beta in dev_inputs:
        d = _lib.DecodeArgs()
        d.base = _scan_args(q, k, v, g, beta, state, state, out, B, None, True, "auto")
        decode_args.append(d)

    def step(i):
        _lib.check(lib.gdn_decode(ctypes.byref(decode_args[i % n_inputs]), stream_handle), "gdn_decode")

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # Timed region: K decode steps back to back with the state carried in
    # place, as config 2 defines its workload (consecutive steps); the 128 MiB
    # state is larger than L2, and each step also drains the write-back the
    # step before it left in L2.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        e0.record()
        for i in range(args.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    own_ms = e0.elapsed_time(e1)
    total_ms = own_ms
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    value = world * DECODE_BYTES * args.steps / (total_ms / 1e3) / 1e9
    mean_ms = total_ms / args.steps
    achieved = DECODE_BYTES / (own_ms / args.steps / 1e3) / 1e9

    # The same launches one at a time, L2 flushed before each (per-launch
    # figure with no write-back of an earlier step inside the kernel's time).
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush_w.fill_(i & 0xFF)
        flush_r.sum()
        starts[i].record()
        step(i)
        ends[i].record()
    torch.cuda.synchronize()
    flushed_ms = statistics.mean(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))

    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 state / bf16 q,k,v",
        "data": "synthetic (seeded; config 2 value distributions)",
        "config": {"workload": "decode, config 2: B=64 sequences x 1 token per rank, 16/32 heads, d=128, "
                               "fp32 state [64,32,128,128] carried in place, steps back to back",
                   "global_batch": B * world, "seq_len": 1, "parallelism": f"sequence-sharded x{world}",
                   "l2": "not flushed: the 128 MiB state is larger than L2 and every step reads and rewrites "
                         "all of it (the flushed per-launch figure is under roofline.flushed)"},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": DECODE_NCU_TRAFFIC,
                     "traffic_source": DECODE_NCU_SOURCE,
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "bytes_per_launch": DECODE_BYTES, "kernel": "decode_kernel<128, bf16>",
                     "timing": "back-to-back launches, one event pair around the timed region / K",
                     "flushed": {"ms_per_launch": flushed_ms,
                                 "achieved": DECODE_BYTES / (flushed_ms / 1e3) / 1e9,
                                 "frac": DECODE_BYTES / (flushed_ms / 1e3) / 1e9 / hbm_peak,
                                 "note": "L2 flushed before each launch (256 MiB write, then 256 MiB read); "
                                         "part of each launch's state write-back leaves L2 after it ends"}},
        "clocks": sampler.summary(),
    }

    if not args.no_extras:
        # --- end to end through the public API with host buffers ---------
        # One pinned staging buffer per step's inputs (q, k, v, g, beta packed at
        # 256-byte offsets) and one device buffer they land in: a step is one
        # H2D copy, the decode call on views of it, one D2H copy of y.
        steps_in = [decode_step_inputs(rank * 1000 + 500 + i) for i in range(n_inputs)]
        offs, total = [], 0
        for x in steps_in[0]:
            offs.append(total)
            total += (x.numel() * x.element_size() + 255) // 256 * 256
        host = []
        for xs in steps_in:
            buf = torch.empty(total, dtype=torch.uint8).pin_memory()
            for x, o in zip(xs, offs):
                nb = x.numel() * x.element_size()
                buf[o:o + nb].copy_(x.contiguous().view(-1).view(torch.uint8))
            host.append(buf)
        dev_in = torch.empty(total, dtype=torch.uint8, device=device)
        views = [dev_in[o:o + x.numel() * x.element_size()].view(x.dtype).view(x.shape)
                 for x, o in zip(steps_in[0], offs)]
        y_host = torch.empty(B, HV, D).pin_memory()
        h2d = total
        d2h = y_host.numel() * y_host.element_size()
        stream = torch.cuda.current_stream(device)
        plan = gdn_b200.DecodePlan(*views, state, g_is_log=True)  # the decode call, prepared once

        def e2e_step(i):
            dev_in.copy_(host[i % n_inputs], non_blocking=True)
            y_host.copy_(plan.run(), non_blocking=True)
            stream.synchronize()  # the step's result is on the host
            return y_host

        for i in range(args.warmup):
            e2e_step(i)
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            e2e_step(i)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e2e_ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
        line["e2e"] = {"value": world * DECODE_BYTES * args.steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "ms_per_step": e2e_ms / args.steps,
                       "api": "gdn_b200.DecodePlan.run (one pinned host buffer of the step's q, k, v, g, beta -> "
                              "device, decode, y -> pinned host; synchronized every step)"}
        line["gpu_launches"] = 2 * args.steps

        # --- config 3 prefill (secondary metric) --------------------------
        pf_ms, pf_clk = measure_prefill(device, clocks=True)
        pf_tflops = PREFILL_FLOP / (pf_ms / 1e3) / 1e12
        line["prefill"] = {"value": PREFILL_T / (pf_ms / 1e3), "unit": "tok/s", "ms": pf_ms,
                           "config": "config 3: B=1, T=8192, 16/32 heads, d=128, bf16 q/k/v, fp32 state from 0",
                           "achieved_tflops": pf_tflops, "frac_of_bf16_peak": pf_tflops / tc_peak, "algo": "auto",
                           "clocks_under_load": pf_clk,
                           "roofline": {"bound": "tensor", "achieved": pf_tflops, "peak": tc_peak, "unit": "TFLOP/s",
                                        "frac": pf_tflops / tc_peak,
                                        "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops, burst)",
                                        "flop_per_call": PREFILL_FLOP, "bytes_per_call": PREFILL_BYTES,
                                        **PREFILL_NCU}}

        # --- config 4 fused block (secondary) --------------------------------
        blk_ms, blk_tok, blk_clk = measure_block(device, clocks=True)
        blk_flop = (PREFILL_FLOP // PREFILL_T) * blk_tok
        line["block"] = {"value": blk_tok / (blk_ms / 1e3), "unit": "tok/s", "ms": blk_ms,
                         "config": "config 4: fused block, B=8 x T=4096, 16/32 heads, d=128, bf16 mixed "
                                   "projection, conv+norms+gates+scan+gated RMSNorm (two state resets included)",
                         "achieved_tflops": blk_flop / (blk_ms / 1e3) / 1e12,
                         "frac_of_bf16_peak": blk_flop / (blk_ms / 1e3) / 1e12 / tc_peak,
                         "clocks_under_load": blk_clk}
        att = measure_attention(device)
        line["attention"] = {
            "prefill_ms": att["prefill_ms"], "prefill_tflops": att["prefill_tflops"],
            "prefill_frac_of_bf16_peak": att["prefill_tflops"] / tc_peak,
            "decode_us": att["decode_us"], "decode_kv_gbs": att["decode_kv_gbs"],
            "layer_decode_us": att["layer_decode_us"],
            "config": "softmax-attention core (norms, rotary, cache append, grouped-query causal attention, "
                      "gate) at 16/2 heads of 256, rotary 64, bf16: 4,096-token prefill (tcgen05 kernel, "
                      "with the cache set-up); one decode token against 4,096 cached positions (split-key "
                      "mma.sync kernel and the split combine), timed as a CUDA-graph "
                      "replay with the cache resident in L2; layer_decode_us: the whole layer at that "
                      "token (hidden 2,048: fused 4-bit q|gate|k|v GEMV, the core, 4-bit o_proj GEMV)"}
        lay = measure_layer(device)
        line["layer"] = {
            "value": lay["tokens"] / (lay["ms"] / 1e3), "unit": "tok/s", "ms": lay["ms"],
            "in_proj_ms": lay["in_proj_ms"], "block_ms": lay["block_ms"], "out_proj_ms": lay["out_proj_ms"],
            "projection_tflops": lay["gemm_flop"] / ((lay["in_proj_ms"] + lay["out_proj_ms"]) / 1e3) / 1e12,
            "decode_us": measure_layer_decode(device),
            "config": "config 4 as a whole layer: hidden states B=8 x T=4096 x 2048 bf16 in and out; in_proj "
                      "(q|k|v|z|b|a, 12,352 x 2,048) and out_proj (2,048 x 4,096) 4-bit affine, group 64 "
                      "(tcgen05 GEMM with on-the-fly dequantization); the fused block between them; "
                      "decode_us: the same layer (Qwen3_5LinearAttention with a RecurrentCache) at one "
                      "decode token, device time of a CUDA-graph replay"}

        # --- the sharded configurations at this world size -----------------
        line["sharded"] = measure_sharded(world, rank, device)

        # --- CPU baseline (rank 0, N=1 only) --------------------------------
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            steps_cpu, secs = cpu_decode_sample()
            mlx = mlx_probe()
            line["cpu_baseline"] = {
                "value": DECODE_BYTES * steps_cpu / secs / 1e9, "unit": "GB/s", "cores": os.cpu_count() or 1,
                "kind": "port",
                "sample": f"{steps_cpu} decode steps x 64 sequences in {secs:.1f} s: torch-CPU restatement of the "
                          "reference's ops path (qw/gated_delta.py:24-41,93-109), one call per sequence; "
                          f"MLX probe on this host: {mlx}",
                "mlx_probe": mlx,
                "prefill_tok_s": cpu_prefill_sample(),
                "prefill_sample": "the first 512 tokens of a config-3-shaped sequence (16/32 heads of 128, "
                                  "state from N(0, 0.02)), the same restatement, all threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
