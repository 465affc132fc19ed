"""Benchmark of the B200 W4A16 quantized-linear hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configs[1]): one Llama-2-7B decoder layer (q/k/v/o 4096->4096,
gate/up 4096->11008, down 11008->4096), GPTQ W4A16 g128 asym, decode M=1, seeded
synthetic weights and activations with the benchmark's distributions. As run, the
projections that read the same input are merged along N (qkv, o, gate_up, down), as
the reference's Marlin loader merges them. One step = one CUDA graph running four
distinct layer copies back to back (4 x 105 MB packed > the 126 MB L2, so weights
stream from HBM); the metric is step time / 4 in microseconds per layer (lower is
better). With N GPUs every projection is column-sharded N ways and its output slices
are all-gathered inside the kernels over NVLink peer memory (strong scaling: the
layer is fixed).

Alongside: the dominant kernel's roofline (HBM bytes per launch / event-timed launch
duration), an end-to-end number through ``QuantLinear.forward`` with the
host<->device copies in the timed region, the same layer at M=8 and at prefill
M=2048, the input-gradient GEMM, the fused MLP block, Llama-2-13B (act-order) and
70B layers, and the CPU oracle timed on the host cores.
"""
from __future__ import annotations

import argparse
import contextlib
import math
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROJ_ORDER = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]
# The layer as run: projections that read the same input merged along N, as the
# reference's Marlin loader merges them (real_loader_marlin.py:65-79); same weight
# bytes and FLOPs as the 7 separate projections, 4 launches instead of 7.
MERGED_GROUPS = [("qkv_proj", ["q_proj", "k_proj", "v_proj"]), ("o_proj", ["o_proj"]),
                 ("gate_up_proj", ["gate_proj", "up_proj"]), ("down_proj", ["down_proj"])]
GROUP = 128
COPIES = 4
METRIC = "W4A16 layer us & % HBM/tensor roofline (M=1 decode, M=2048 prefill), 1-8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def proj_bytes(K: int, N: int, M: int, act: bool = False) -> int:
    """Algorithmic bytes of one W4A16 call: packed weight, zeros, scales, X and Y."""
    G = K // GROUP
    b = K * N // 2 + G * N // 2 + 2 * G * N + 2 * M * K + 2 * M * N
    return b + (4 * K if act else 0)


def layer_shapes(merged: bool = True, model: str = "7b"):
    """(name, K, N) of one decoder layer's projections: merged (as run) or the 7 separate ones."""
    from drofell_for_revision_b200.synthetic import LLAMA2_7B, LLAMA2_13B, LLAMA2_70B
    table = {"7b": LLAMA2_7B, "13b": LLAMA2_13B, "70b": LLAMA2_70B}[model]
    if not merged:
        return [(p, *table[p]) for p in PROJ_ORDER]
    return [(name, table[parts[0]][0], sum(table[q][1] for q in parts)) for name, parts in MERGED_GROUPS]


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([c.strip() for c in out.stdout.strip().split(",")])
            except Exception:
                return
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=10)

    def summary(self):
        if not self.rows:
            return None
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


# --------------------------------------------------------------------------- CPU legs
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_layer_pass(layers_cpu, xs_cpu, threads, scratch):
    """One decoder layer of the reference's CPU semantics (real_quant.py:69-102): per
    projection the dequant into a dense fp16 W, then the fp32 matmul. Returns the
    seconds spent in each of the two steps."""
    from oracle import w4a16_oracle as orc
    t_dq = t_mm = 0.0
    for (name, K, N), layer, x in zip(layer_shapes(), layers_cpu, xs_cpu):
        w = scratch[: K * N].view(np.float16).reshape(K, N)
        t0 = time.perf_counter()
        orc.c_dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), None, GROUP,
                           threads=threads, out=w)
        t1 = time.perf_counter()
        orc.c_matmul_f16w(x.numpy(), w, threads=threads)
        t2 = time.perf_counter()
        t_dq += t1 - t0
        t_mm += t2 - t1
    return t_dq, t_mm


def cpu_inputs(M: int, seed: int = 0):
    from drofell_for_revision_b200 import synthetic
    layers = [synthetic.make_layer(K, N, GROUP, seed=seed * 100 + i) for i, (_, K, N) in enumerate(layer_shapes())]
    xs = [synthetic.make_activations(M, K, seed=seed * 100 + 50 + i) for i, (_, K, N) in enumerate(layer_shapes())]
    return layers, xs


def time_cpu_oracle(M: int, budget_s: float, threads: int, max_layers: int | None = None):
    """The C oracle (dequant, then fp32 matmul) over a bounded sample of whole layers:
    (median seconds per layer, median dequant seconds, median matmul seconds, layers)."""
    layers, xs = cpu_inputs(M)
    scratch = np.empty(max(K * N for _, K, N in layer_shapes()), dtype=np.uint16)
    cpu_layer_pass(layers, xs, threads, scratch)  # warm-up
    dq, mm = [], []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end and (max_layers is None or len(dq) < max_layers)) or not dq:
        a, b = cpu_layer_pass(layers, xs, threads, scratch)
        dq.append(a)
        mm.append(b)
    tot = [a + b for a, b in zip(dq, mm)]
    return statistics.median(tot), statistics.median(dq), statistics.median(mm), len(tot)


def base_config(world: int) -> dict:
    """The workload both arms measure (benchmark configs[1])."""
    return {"workload": "llama2-7b-layer-decode-m1",
            "projections": [f"{n} ({'+'.join(p)})" for n, p in MERGED_GROUPS], "M": 1, "group_size": GROUP,
            "act_order": False, "n_gpus": world}


def cpu_baseline_entry(sec, dq, mm, reps, threads):
    return {"value": round(sec * 1e6, 1), "unit": "us/layer", "cores": threads, "kind": "port",
            "dequant_us": round(dq * 1e6, 1), "matmul_us": round(mm * 1e6, 1), "cpu_model": cpu_model(),
            "sample": (f"median of {reps} full Llama-2-7B decoder layers (its 7 projections as 4 merged matmuls, "
                       f"M=1): C oracle dequant (real_quant.py:69-90 semantics) then fp32 matmul, "
                       f"{threads} OpenMP threads")}


def run_reference_arm(args, rank: int, world: int):
    """The reference's CPU dequant+matmul semantics (oracle port, all host threads)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # a bounded sample: at most args.steps layers, or about cpu_budget x 6 seconds
    budget_s = max(args.cpu_budget * 6, 30.0)
    t0 = time.perf_counter()
    sec, dq, mm, done = time_cpu_oracle(1, budget_s, threads, max_layers=args.steps)
    us = sec * 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 3), "unit": "us/layer", "n_gpus": world,
        "steps": done, "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic", "config": base_config(world),
        "cpu_baseline": cpu_baseline_entry(sec, dq, mm, done, threads),
        "e2e": {"value": round(us, 3), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(time.perf_counter() - t0, 1),
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
def graph_time_per_launch(fn, launches: int, warm_s: float = 0.3, timed_s: float = 0.05, sampler=None) -> float:
    """Average device time (ms) of one ``fn(i)`` call: ``launches`` calls are captured
    in one CUDA graph, replayed for ``warm_s`` seconds so the SM clocks have ramped up,
    then replayed for at least ``timed_s`` seconds between CUDA events. Host launch
    latency is not part of the number (inter-kernel gaps on the GPU are). ``sampler``
    (a ClockSampler) is entered around the timed replays."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            fn(i)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < warm_s:
        g.replay()
        torch.cuda.synchronize()
    start.record()
    g.replay()
    end.record()
    torch.cuda.synchronize()
    reps = max(3, int(math.ceil(timed_s * 1e3 / max(start.elapsed_time(end), 1e-3))))
    ctx = sampler if sampler is not None else contextlib.nullcontext()
    with ctx:
        start.record()
        for _ in range(reps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / (reps * launches)
    del g
    return ms


def build_layers(device, rank, world, copies, seed0=0, peer=None, shapes=None, local_shards=False, max_m=16,
                 act=False):
    """copies x the layer's QuantLinears (column shard of this rank), from CPU-generated
    tensors. With ``peer`` (N > 1) every M <= ``max_m`` runs with the all-gather fused
    into the kernel. ``local_shards``: each rank generates only its own columns (large
    models)."""
    from drofell_for_revision_b200 import synthetic
    from drofell_for_revision_b200.exllama import CacheV2, TuningParams
    from drofell_for_revision_b200.real_quant import QuantLinear
    from drofell_for_revision_b200.sharded import ShardedQuantLinear
    tp, cache = TuningParams(), CacheV2(device)
    shapes = shapes or layer_shapes()
    out = []
    for c in range(copies):
        mods = []
        for i, (name, K, N) in enumerate(shapes):
            seed = (seed0 + c) * 100 + i
            if local_shards:
                layer = synthetic.make_layer(K, N // world, GROUP, seed=seed * 16 + rank)
                lin = QuantLinear(GROUP, K, N // world, False, False)
                lin.qweight.copy_(layer.qweight)
                lin.qzeros.copy_(layer.qzeros)
                lin.scales.copy_(layer.scales)
                lin = lin.to(device)
                lin.post_init(tp, cache)
                mods.append(ShardedQuantLinear(lin, N, rank, world, peer=peer, max_m=max_m))
            else:
                layer = synthetic.make_layer(K, N, GROUP, act_order=act, seed=seed)
                mods.append(ShardedQuantLinear.from_packed(layer.qweight, layer.qzeros, layer.scales, layer.g_idx,
                                                           GROUP, act, rank, world, device, tuning_params=tp,
                                                           cache=cache, peer=peer, max_m=max_m))
        out.append(mods)
    return out


def make_inputs(M, device, seed=0, dtype=torch.float16, shapes=None):
    from drofell_for_revision_b200 import synthetic
    return [synthetic.make_activations(M, K, seed=seed * 100 + 50 + i, dtype=dtype).to(device)
            for i, (_, K, N) in enumerate(shapes or layer_shapes())]


def capture_step_graphs(layer_copies, xs, stream):
    """One CUDA graph that runs every layer copy once, back to back: one step is a decode
    pass through a stack of len(layer_copies) layers (a model's forward is one graph).
    The copies hold different weights, so the stack streams more than L2 holds."""
    with torch.cuda.stream(stream):
        for mods in layer_copies:  # warm-up (allocator, workspace) outside capture
            for m, x in zip(mods, xs):
                m(x)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        outs = [[m(x) for m, x in zip(mods, xs)] for mods in layer_copies]
    return [g], outs


def timed_replays(graphs, steps, warmup, world, warm_s: float = 0.3):
    """``warmup`` untimed replays, more until ``warm_s`` seconds have passed (SM clocks
    ramp up under sustained load), then exactly ``steps`` timed replays (ms per step)."""
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    # The extra warm-up is a replay COUNT agreed by all ranks (the graphs hold NCCL
    # collectives, so every rank must replay them the same number of times).
    t0 = time.perf_counter()
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    per = max(time.perf_counter() - t0, 1e-6) / len(graphs)
    extra = int(math.ceil(warm_s / per))
    if world > 1:
        t = torch.tensor([extra], dtype=torch.int64, device=torch.device("cuda", torch.cuda.current_device()))
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        extra = int(t.item())
    for i in range(extra):
        graphs[i % len(graphs)].replay()
        if (i + 1) % 64 == 0:
            torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for i in range(steps):
        graphs[i % len(graphs)].replay()
        ev[i + 1].record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    timed_replays.last_median = statistics.median(per)
    return ev[0].elapsed_time(ev[steps]) / steps  # ms per step (mean over the K timed steps)


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def dominant_kernel_timing(device, launches=64):
    """Device time per launch of the largest decode projection (merged gate_up
    4096->22016, M=1, the path PATH_AUTO picks) rotating 8 weight copies (360 MB > L2), from a
    CUDA graph of ``launches`` back-to-back launches. Returns (avg ms, plan, bytes)."""
    from drofell_for_revision_b200 import _capi, synthetic
    K, N = 4096, 22016  # gate_up_proj, the layer's largest launch
    handles, keep = [], []
    for c in range(8):
        layer = synthetic.make_layer(K, N, GROUP, seed=900 + c)
        qw, qz, sc = layer.qweight.to(device), layer.qzeros.to(device), layer.scales.to(device)
        keep.append((qw, qz, sc))
        handles.append(_capi.Handle(qw, qz, sc, None, device.index))
    x = synthetic.make_activations(1, K, seed=5).to(device)
    y = torch.empty((1, N), dtype=torch.float16, device=device)
    ws = torch.empty(max(1, handles[0].workspace_size(1, torch.float16)), dtype=torch.uint8, device=device)
    ms = graph_time_per_launch(lambda i: handles[i % 8].gemm(x, y, _capi.PATH_AUTO, ws), launches)
    plan = handles[0].plan(1)
    return ms, plan, proj_bytes(K, N, 1)


def e2e_public_api(layer_copies, M, steps, warmup, device, world):
    """Per step, the same decoder-layer stack as the device-timed value (every layer copy
    once), through the public API (eager QuantLinear.forward) on a layer's dataflow: the
    stack's input X from pinned host memory to the device; per layer qkv_proj, o_proj on
    the first 4096 qkv outputs (a view standing in for attention), gate_up_proj, down_proj
    on the first 11008 gate_up outputs (standing in for SiLU x mul), whose output feeds the
    next layer; the stack's output back to pinned host memory. Returns ms per layer."""
    shapes = layer_shapes()
    assert [n for n, _, _ in shapes] == ["qkv_proj", "o_proj", "gate_up_proj", "down_proj"]
    x_h = torch.randn((M, shapes[0][1]), dtype=torch.float32).half().pin_memory()
    y_h = torch.empty((M, shapes[-1][2]), dtype=torch.float16).pin_memory()

    # the modules a user calls: QuantLinear itself on one GPU, the column-sharded wrapper on several
    mods = [[m.local if world == 1 else m for m in copy] for copy in layer_copies]
    n_o, n_down = shapes[1][1], shapes[3][1]

    def step():
        h = x_h.to(device, non_blocking=True)
        for qkv, o, gate_up, down in mods:
            h = o(qkv(h)[:, :n_o])
            h = down(gate_up(h)[:, :n_down])
        y_h.copy_(h, non_blocking=True)

    for _ in range(warmup):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    return s.elapsed_time(e) / steps / len(mods), x_h.numel() * 2, y_h.numel() * 2


def count_launches(layer_copies, M, world):
    """Kernels of this library per layer step: GEMV passes or the GEMM (+ its split-K
    reduction), the act-order X gather, and with the fused all-gather the signal kernel."""
    from drofell_for_revision_b200 import _capi
    n = 0
    for m in layer_copies[0]:
        h = m.local.q4_matrix._h
        plan = h.plan(M)
        if plan[0] in (_capi.KERN_GEMV, _capi.KERN_GEMV_MMA):
            n += (M + plan[3] - 1) // plan[3]
        else:
            n += 1 + (1 if plan[0] == _capi.KERN_EXACT and plan[2] > 1 else 0)
        n += 1 if h._g_idx_host is not None else 0
        n += 1 if (world > 1 and getattr(m, "_y_full", None) is not None and M <= m.max_m) else 0
    return n


def model_layer_lines(device, stream, model: str, act: bool, Ms, steps: int, warmup: int, peaks: dict) -> dict:
    """One merged decoder layer of ``model`` at each M on this GPU (benchmark configs 4 and
    5): us per layer through the public module API in a CUDA graph (mean over the timed
    replays, the median replay beside it), with the HBM fraction (weights + activations)
    and the tensor fraction (2 M N K) beside it."""
    shapes = layer_shapes(model=model)
    lb = sum(proj_bytes(K, N, 1, act) for _, K, N in shapes)
    copies = max(1, -(-300_000_000 // lb))  # the stack exceeds L2
    layers = build_layers(device, 0, 1, copies, seed0=70 if act else 80, shapes=shapes, max_m=16, act=act)
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    tc = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    out = {"workload": f"llama2-{model}-layer" + ("-act-order" if act else ""), "layer_copies": copies,
           "projections": [f"{n} {K}->{N}" for n, K, N in shapes]}
    for M in Ms:
        xs = make_inputs(M, device, seed=M, shapes=shapes)
        graphs, _ = capture_step_graphs(layers, xs, stream)
        n = max(3, min(steps, 200 if M <= 16 else 50))
        ms = timed_replays(graphs, n, warmup, 1) / len(layers)
        ms_med = timed_replays.last_median / len(layers)
        del graphs
        b = sum(proj_bytes(K, N, M, act) for _, K, N in shapes)
        f = sum(2 * M * K * N for _, K, N in shapes)
        out[f"M={M}"] = {"us": round(ms * 1e3, 2), "us_median": round(ms_med * 1e3, 2),
                         "hbm_gbs": round(b / (ms * 1e-3) / 1e9, 1),
                         "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 4),
                         "tflops": round(f / (ms * 1e-3) / 1e12, 1), "frac_tensor": round(f / (ms * 1e-3) / 1e12 / tc, 4)}
    del layers
    torch.cuda.synchronize()
    return out


def fused_mlp_line(device, Ms, peaks: dict) -> dict:
    """The Llama-2-7B decode MLP block, RMSNorm -> gate/up -> SiLU x mul -> down, at each
    M: the fused entry point (w4a16_mlp_forward: two launches at M <= 2) beside the same
    block as five separate kernels (RMSNorm, gate, up, SiLU x mul, down), which is the
    reference's chain (fuse_v2/q_mlp.cu:96-133). CUDA graphs over rotated weight copies
    larger than L2."""
    from drofell_for_revision_b200 import _capi, synthetic
    K, I = 4096, 11008
    blk_bytes = 2 * proj_bytes(K, I, 1) + proj_bytes(I, K, 1)
    copies = max(2, -(-300_000_000 // blk_bytes))
    blocks = []
    for c in range(copies):
        hs = []
        for j, (k, n) in enumerate(((K, I), (K, I), (I, K))):
            lay = synthetic.make_layer(k, n, GROUP, seed=900 + 10 * c + j)
            hs.append(_capi.Handle(lay.qweight.to(device), lay.qzeros.to(device), lay.scales.to(device), None,
                                   device.index))
        blocks.append(hs)
    norm_w = (1.0 + 0.1 * torch.randn(K)).half().to(device)
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    out = {"workload": "llama2-7b-mlp-block", "block": f"RMSNorm {K}, gate/up {K}->{I}, SiLU x mul, down {I}->{K}",
           "block_copies": copies}
    for M in Ms:
        x = synthetic.make_activations(M, K, seed=M + 3).to(device)
        y = torch.empty((M, K), dtype=torch.float16, device=device)
        r = torch.empty((M, K), dtype=torch.float16, device=device)
        g = torch.empty((M, I), dtype=torch.float16, device=device)
        u = torch.empty((M, I), dtype=torch.float16, device=device)

        def fused(i):
            gh, uh, dh = blocks[i % copies]
            _capi.mlp_forward(gh, uh, dh, norm_w, 1e-5, x, y, r, g, u)

        def chain(i):
            gh, uh, dh = blocks[i % copies]
            _capi.rms_norm(x, norm_w, 1e-5, r)
            gh.gemm(r, g)
            uh.gemm(r, u)
            _capi.silu_mul(g, u, g)
            dh.gemm(g, y)

        b = 2 * proj_bytes(K, I, M) + proj_bytes(I, K, M)
        res = {}
        for name, fn in (("fused", fused), ("five_kernels", chain)):
            ms = graph_time_per_launch(fn, copies * 4, timed_s=0.1)
            res[name] = {"us": round(ms * 1e3, 2), "hbm_gbs": round(b / (ms * 1e-3) / 1e9, 1),
                         "frac_hbm": round(b / (ms * 1e-3) / 1e9 / hbm, 4)}
        out[f"M={M}"] = res
    for hs in blocks:
        for h in hs:
            h.close()
    torch.cuda.synchronize()
    return out


def backward_line(layer_copies, device, M: int, peaks: dict) -> dict:
    """The input gradient dX = dY W^T of the merged 7B layer at M tokens on the tcgen05
    transposed GEMM (w4a16_gemm_t), graph-replayed over the layer copies."""
    hs = [[m.local.q4_matrix._h for m in mods] for mods in layer_copies]
    shapes = layer_shapes()
    dys = [torch.randn((M, N), device=device).half() for _, K, N in shapes]
    dxs = [torch.empty((M, K), dtype=torch.float16, device=device) for _, K, N in shapes]
    wss = [torch.empty(max(1, hs[0][i].workspace_size_t(M, torch.float16)), dtype=torch.uint8, device=device)
           for i in range(len(shapes))]

    def fn(i):
        for j, h in enumerate(hs[i % len(hs)]):
            h.gemm_t(dys[j], dxs[j], wss[j])

    ms = graph_time_per_launch(fn, len(hs), timed_s=0.3)
    f = sum(2 * M * K * N for _, K, N in shapes)
    tc = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    return {"workload": f"llama2-7b-layer-input-grad-m{M}", "us": round(ms * 1e3, 2),
            "tflops": round(f / (ms * 1e-3) / 1e12, 1), "frac_of_bf16_peak": round(f / (ms * 1e-3) / 1e12 / tc, 4),
            "note": "dX = dY W^T for qkv, o, gate_up, down (w4a16_gemm_t; the reference reconstructs W and runs "
                    "cublasHgemm OP_T)"}


def run_ours(args, rank: int, world: int, local_rank: int):
    from drofell_for_revision_b200 import _capi
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _capi.lib()
    peaks, peaks_kind = load_peaks()
    stream = torch.cuda.Stream(device)

    peer = None
    if world > 1:
        from drofell_for_revision_b200.sharded import PeerGather
        peer = PeerGather(rank, world, device)
    # sharded: decode and the M = 2048 prefill both run with the all-gather fused in
    layer_copies = build_layers(device, rank, world, COPIES, peer=peer, max_m=2048 if world > 1 else 16)
    xs = make_inputs(1, device)
    graphs, _ = capture_step_graphs(layer_copies, xs, stream)

    with ClockSampler(local_rank) as clk:
        ms_step = timed_replays(graphs, args.steps, args.warmup, world)
    ms_median = max_over_ranks(timed_replays.last_median, world, device)
    ms_step = max_over_ranks(ms_step, world, device)
    ms_layer = ms_step / len(layer_copies)  # one step = the stack of layer copies
    clocks = clk.summary()

    launches_per_step = count_launches(layer_copies, 1, world) * len(layer_copies)
    gpu_launches = launches_per_step * args.steps

    # with N GPUs: the same stack on this rank's column shards alone, without the
    # all-gather: the compute side of the scaling, reported beside the gathered value
    ms_local = None
    if world > 1:
        local_copies = [[m.local for m in mods] for mods in layer_copies]
        graphs_l, _ = capture_step_graphs(local_copies, xs, stream)
        ms_local = max_over_ranks(timed_replays(graphs_l, args.steps, args.warmup, world), world, device) / len(
            layer_copies)
        del graphs_l
    # the same layer at M = 8 (the benchmark's second decode size: the mma.sync GEMV)
    graphs8, _ = capture_step_graphs(layer_copies, make_inputs(8, device, seed=8), stream)
    ms8 = max_over_ranks(timed_replays(graphs8, max(3, min(args.steps, 500)), args.warmup, world), world,
                         device) / len(layer_copies)
    del graphs8
    # the same layer as 7 separate projections (7 launches; reported beside the value)
    del graphs
    torch.cuda.synchronize()
    shapes7 = layer_shapes(merged=False)
    copies7 = build_layers(device, rank, world, COPIES, seed0=50, peer=peer, shapes=shapes7)
    graphs7, _ = capture_step_graphs(copies7, make_inputs(1, device, shapes=shapes7), stream)
    ms7 = max_over_ranks(timed_replays(graphs7, args.steps, args.warmup, world), world, device) / len(copies7)
    del graphs7, copies7
    # Llama-2-70B layer (the multi-GPU configuration): this rank's column shards only
    shapes70 = layer_shapes(model="70b")
    bytes70 = sum(proj_bytes(K, N, 1) for _, K, N in shapes70)
    copies70 = max(1, -(-300_000_000 * world // bytes70))  # > L2 per GPU
    layers70 = build_layers(device, rank, world, copies70, seed0=90, peer=peer, shapes=shapes70, local_shards=True)
    graphs70, _ = capture_step_graphs(layers70, make_inputs(1, device, shapes=shapes70), stream)
    steps70 = max(3, min(args.steps, 300))
    ms70 = max_over_ranks(timed_replays(graphs70, steps70, args.warmup, world), world, device) / len(layers70)
    del graphs70, layers70
    torch.cuda.synchronize()
    graphs = None

    # dominant kernel roofline (1-GPU shapes; every rank measures its own GPU)
    avg_ms, plan, bytes_per_launch = dominant_kernel_timing(device)
    achieved = bytes_per_launch / (avg_ms * 1e-3) / 1e9
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("gemv_gate_up_4096x22016_m1_bytes_per_launch")
        except ValueError:
            traffic = None

    # e2e through the public API with host copies
    e2e_ms, h2d, d2h = e2e_public_api(layer_copies, 1, args.steps, args.warmup, device, world)
    e2e_ms = max_over_ranks(e2e_ms, world, device)

    # prefill M=2048 on the tensor-core path (same layer copies)
    torch.cuda.synchronize()
    xs_p = make_inputs(2048, device, seed=7)
    graphs_p, _ = capture_step_graphs(layer_copies, xs_p, stream)
    p_steps = max(3, min(args.steps, 20))
    ms_p = timed_replays(graphs_p, p_steps, max(3, args.warmup), world)
    ms_p = max_over_ranks(ms_p, world, device) / len(layer_copies)
    flops = sum(2 * 2048 * K * N for _, K, N in layer_shapes())
    tflops = flops / (ms_p * 1e-3) / 1e12
    del graphs_p

    extra = {}
    if world == 1 and not args.quick:
        extra["backward"] = backward_line(layer_copies, device, 2048, peaks)
        extra["fused_mlp"] = fused_mlp_line(device, (1, 8), peaks)
        extra["llama2_13b_act_order"] = model_layer_lines(device, stream, "13b", True, (1, 128, 1024), args.steps,
                                                          args.warmup, peaks)
        extra["llama2_70b"] = model_layer_lines(device, stream, "70b", False, (1, 16, 128, 2048), args.steps,
                                                args.warmup, peaks)

    layer_bytes = sum(proj_bytes(K, N, 1) for _, K, N in layer_shapes())
    us = ms_layer * 1e3
    line = {
        "metric": METRIC, "value": round(us, 3), "unit": "us/layer", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic",
        "config": base_config(world),
        "method": {"parallelism": (f"column-shard x{world}: the all-gather fused into the kernel over NVLink peer "
                                   f"memory (decode GEMV; prefill tcgen05 GEMM epilogue)") if world > 1
                                  else "single GPU",
                   "l2": f"{COPIES} rotated layer copies, {COPIES * layer_bytes / 1e6:.0f} MB > 126 MB L2",
                   "timing": (f"one CUDA graph per step running the {len(layer_copies)} rotated layer copies back to "
                              f"back (a {len(layer_copies)}-layer decode stack; a model's forward is one graph); "
                              f"us/layer = step time / {len(layer_copies)}; CUDA events, max over ranks"),
                   "layers_per_step": len(layer_copies)},
        "ms_per_step_median": round(ms_median, 5),
        "layer_hbm_gbs": round(layer_bytes / world / (ms_layer * 1e-3) / 1e9, 1),
        "layer_m8": {"value": round(ms8 * 1e3, 3), "unit": "us/layer", "M": 8,
                     "hbm_gbs": round(sum(proj_bytes(K, N, 8) for _, K, N in layer_shapes()) / world / (ms8 * 1e-3) / 1e9, 1),
                     "note": "the same 4-layer stack at decode M = 8 (GEMV on mma.sync)"},
        **({"layer_without_gather": {"value": round(ms_local * 1e3, 3), "unit": "us/layer",
                                     "note": "this rank's column shards of the same stack, no all-gather "
                                             "(max over ranks)"}} if ms_local is not None else {}),
        "layer_7_launches": {"value": round(ms7 * 1e3, 3), "unit": "us/layer",
                             "note": "q, k, v, o, gate, up, down as 7 separate projections"},
        "llama2_70b_layer": {"value": round(ms70 * 1e3, 3), "unit": "us/layer", "M": 1,
                             "hbm_gbs_per_gpu": round(bytes70 / world / (ms70 * 1e-3) / 1e9, 1),
                             "layer_copies": copies70,
                             "note": "merged 70B projections, column shard of this rank (the multi-GPU config)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "peak_kind": peaks_kind,
                     "kernel": f"{KERNEL_NAMES.get(plan[0], plan[0])} (family {plan[0]}, tile {plan[1]}, "
                               f"splits {plan[2]}, mode {plan[3]}) gate_up_proj 4096x22016 M=1",
                     "bytes_per_launch": bytes_per_launch, "avg_launch_us": round(avg_ms * 1e3, 3),
                     "timing": "CUDA graph of 64 back-to-back launches over 8 weight copies (360 MB > L2)"},
        "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "api": (f"QuantLinear.forward (eager) on the same {len(layer_copies)}-layer stack as the value, one step per "
                        f"token: pinned host X -> per layer qkv -> o -> gate_up -> down -> pinned host Y (slices "
                        f"of the previous output stand in for attention and SiLU x mul); us/layer = step time / "
                        f"{len(layer_copies)}")},
        "prefill": {"workload": "llama2-7b-layer-prefill-m2048", "value": round(ms_p * 1e3, 2), "unit": "us/layer",
                    "tflops": round(tflops, 1),
                    "frac_of_bf16_peak": round(tflops / float(peaks.get("bf16_tflops_sustained",
                                                                          FALLBACK_PEAKS["bf16_tflops_sustained"])), 4),
                    "peak": "bf16_tflops_sustained", "peak_kind": peaks_kind},
        "gpu_launches": gpu_launches,
        "clocks": clocks,
        **extra,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sec, dq, mm, reps = time_cpu_oracle(1, args.cpu_budget, threads)
        line["cpu_baseline"] = cpu_baseline_entry(sec, dq, mm, reps, threads)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if peer is not None:
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        peer.close()


KERNEL_NAMES = {1: "gemv (CUDA cores)", 2: "tcgen05 decode pass", 3: "tcgen05 exact-W GEMM",
                4: "gemv (mma.sync on the repacked weight)"}

CASES = {
    # name: (K, N, M, path, dtype, act_order)
    "gemv_gate_m1": (4096, 11008, 1, 1, "fp16", False),
    "gemv_q_m1": (4096, 4096, 1, 1, "fp16", False),
    "gemv_down_m1": (11008, 4096, 1, 1, "fp16", False),
    "gemv_gate_m4": (4096, 11008, 4, 1, "fp16", False),
    "gemv_70b_gate_m1": (8192, 28672, 1, 1, "fp16", False),
    "gemv_gate_m1_bf16": (4096, 11008, 1, 1, "bf16", False),
    "gemv_gate_up_m1": (4096, 22016, 1, 1, "fp16", False),
    "gemv_qkv_m1": (4096, 12288, 1, 1, "fp16", False),
    "gemv_70b_down_m1": (28672, 8192, 1, 1, "fp16", False),
    "gemv_gate_m8": (4096, 11008, 8, 1, "fp16", False),
    "gemv_gate_up_m8": (4096, 22016, 8, 1, "fp16", False),
    "gemv_70b_gate_m16": (8192, 28672, 16, 1, "fp16", False),
    "tc_gate_m1": (4096, 11008, 1, 2, "fp16", False),
    "tc_q_m1": (4096, 4096, 1, 2, "fp16", False),
    "tc_down_m1": (11008, 4096, 1, 2, "fp16", False),
    "tc_70b_gate_m1": (8192, 28672, 1, 2, "fp16", False),
    "tc_70b_kv_m1": (8192, 1024, 1, 2, "fp16", False),
    "tc_gate_m8": (4096, 11008, 8, 2, "fp16", False),
    "tc_gate_m16": (4096, 11008, 16, 2, "fp16", False),
    "tc_gate_m128": (4096, 11008, 128, 2, "fp16", False),
    "tc_70b_gate_m128": (8192, 28672, 128, 2, "fp16", False),
    "tc_gate_m2048": (4096, 11008, 2048, 2, "fp16", False),
    "tc_q_m2048": (4096, 4096, 2048, 2, "fp16", False),
    "tc_act13b_m1024": (5120, 13824, 1024, 2, "fp16", True),
    "tc_70b_gate_m2048": (8192, 28672, 2048, 2, "fp16", False),
    "dequant_gate": (4096, 11008, 0, -1, "fp16", False),
    # per-rank column shards of the merged 7B layer at prefill (4 and 8 GPUs)
    "tc_qkv_m2048": (4096, 12288, 2048, 2, "fp16", False),
    "tc_gate_up_m2048": (4096, 22016, 2048, 2, "fp16", False),
    "tc_down_m2048": (11008, 4096, 2048, 2, "fp16", False),
    "tc_qkv_s4_m2048": (4096, 3072, 2048, 2, "fp16", False),
    "tc_o_s4_m2048": (4096, 1024, 2048, 2, "fp16", False),
    "tc_gate_up_s4_m2048": (4096, 5504, 2048, 2, "fp16", False),
    "tc_down_s4_m2048": (11008, 1024, 2048, 2, "fp16", False),
    "tc_qkv_s8_m2048": (4096, 1536, 2048, 2, "fp16", False),
    "tc_o_s8_m2048": (4096, 512, 2048, 2, "fp16", False),
    "tc_gate_up_s8_m2048": (4096, 2752, 2048, 2, "fp16", False),
    "tc_down_s8_m2048": (11008, 512, 2048, 2, "fp16", False),
}


def run_case(name: str, launches: int, eager: bool = False) -> None:
    """One kernel family on one shape, event-timed per launch; weights rotate over
    enough copies to exceed L2. For ncu captures and sweeps, not a bench line."""
    from drofell_for_revision_b200 import _capi, synthetic
    K, N, M, path, dt, act = CASES[name]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    wbytes = K * N // 2
    copies = max(1, min(8, (300 * 2**20) // max(1, wbytes) + 1))
    handles, keep = [], []
    for c in range(copies):
        layer = synthetic.make_layer(K, N, GROUP, act_order=act, seed=1000 + c)
        t = (layer.qweight.to(device), layer.qzeros.to(device), layer.scales.to(device))
        keep.append(t)
        handles.append(_capi.Handle(*t, layer.g_idx if act else None, 0))
    dtype = torch.float16 if dt == "fp16" else torch.bfloat16
    if path == -1:
        out = torch.empty((K, N), dtype=dtype, device=device)
        fn = lambda i: handles[i % copies].dequant(out)  # noqa: E731
        nbytes = K * N // 2 + (K // GROUP) * N // 2 + 2 * (K // GROUP) * N + 2 * K * N
        flops = 0
    else:
        x = synthetic.make_activations(M, K, seed=3, dtype=dtype).to(device)
        y = torch.empty((M, N), dtype=dtype, device=device)
        ws = torch.empty(max(1, handles[0].workspace_size(M, dtype, path)), dtype=torch.uint8, device=device)
        fn = lambda i: handles[i % copies].gemm(x, y, path, ws)  # noqa: E731
        nbytes = proj_bytes(K, N, M, act)
        flops = 2 * M * N * K
    if eager:  # a few plain launches and nothing else: the shape an ncu capture wants
        for i in range(launches):
            fn(i)
        torch.cuda.synchronize()
        print(json.dumps({"case": name, "eager_launches": launches}), flush=True)
        return
    sampler = ClockSampler(0)
    avg = graph_time_per_launch(fn, launches, timed_s=0.6, sampler=sampler)
    res = {"case": name, "K": K, "N": N, "M": M, "path": path, "copies": copies, "launches": launches,
           "avg_us": round(avg * 1e3, 3), "gbs": round(nbytes / (avg * 1e-3) / 1e9, 1),
           "tflops": round(flops / (avg * 1e-3) / 1e12, 2) if flops else None,
           "plan": list(handles[0].plan(max(M, 1), dtype, max(path, 0))) if path >= 0 else None,
           "clocks": sampler.summary()}
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(CASES), default=None,
                    help="time one kernel on one shape instead of the benchmark")
    ap.add_argument("--launches", type=int, default=50)
    ap.add_argument("--eager", action="store_true", help="--case only: plain launches, no timing (for ncu)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="skip the 13B / 70B configuration and backward lines")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.case:
        run_case(args.case, args.launches, args.eager)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.cuda.synchronize()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
