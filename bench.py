#!/usr/bin/env python
"""Benchmark of the routed-expert int4 MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl wisp|reference]

Default workload (the configuration its metric is
quoted on at 1/2/4/8 GPUs): a stack of 4 MoE layers, 384 routed experts + 1
shared expert, hidden 7168, moe_intermediate 2048, softmax top-8, int4 group
128 weights, 256 decode tokens per step, bf16 activations, seed 3. A step is
one pass of the 256 tokens through the 4 layers (router, dispatch, grouped
gate/up + SwiGLU, grouped down + weighted combine; between layers the output
is RMS-rescaled to the next layer's bf16 input). With N GPUs the routed
experts are sharded N ways and tokens are exchanged with NCCL all-to-all
(strong scaling: the total work is fixed).

The metric is MoE-layer tokens/s = tokens x layers per second (whole job).
Every step streams ~35 GB of expert weights, far larger than the 126 MB L2,
so no flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s; int4 weight GB/s vs 8 TB/s HBM at 1/2/4/8 B200"
UNIT = "tokens/s"


# DRAM bytes (read + write) per algorithmic byte of one grouped-FFN call,
# from an ncu capture of the ep_profile workload (1,507.4 MB of traffic for
# 1,476.03 MB of int4 weights and scales, profiles/grouped_ffn_ep_profile_traffic.md):
# the full-size layer is too large for a multi-pass capture, and its traffic
# grows with the experts streamed.
TRAFFIC_PER_ALGORITHMIC_BYTE = 1507.58 / 1476.03


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"unavailable": "nvidia-smi not runnable"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"unavailable": "no samples"}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# Reference CPU path (the reference engine's own compiled C code)
# ---------------------------------------------------------------------------

def _cpu_sample_setup(spec, n_blobs: int = 16, seed: int = 0):
    """Host-side inputs for the reference CPU path: the fp16 router of the
    configuration's shape and n_blobs distinct expert blobs addressed
    cyclically by expert id (timing only; parity is tested in tests/)."""
    import numpy as np
    from wisp_b200.blob import Int4Matrix, pack_blob

    rng = np.random.default_rng(seed)
    M, I, gs = spec.hidden, spec.inter, spec.group_size

    def mat(rows, cols):
        n = rows * cols
        return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                          None, rows, cols)

    blobs = [np.frombuffer(pack_blob(mat(I, M), mat(I, M), mat(M, I), gs), np.uint8)
             for _ in range(n_blobs)]
    router = np.float16(rng.standard_normal((spec.n_experts, M)) * 0.02).view(np.uint16)
    xs = [rng.standard_normal(M).astype(np.float32) for _ in range(8)]
    return router, blobs, xs


def _cpu_token_time(ref, spec, router, blobs, xs, n_tokens: int) -> float:
    """Seconds for n_tokens single-token passes through one layer."""
    E = spec.n_experts
    table = [blobs[e % len(blobs)] for e in range(E)]
    shared = blobs[-1] if spec.has_shared else None
    t0 = time.perf_counter()
    for i in range(n_tokens):
        ref.moe_token(router, None, xs[i % len(xs)], spec.top_k, table, shared)
    return time.perf_counter() - t0


def cpu_baseline(spec, budget_s: float = 12.0) -> dict:
    from oracle.oracle import RefCPU
    if not RefCPU.available():
        return {"unavailable": "oracle/_ref/libwisp_ref.so not built"}
    ref = RefCPU(threads=RefCPU.host_cores())
    router, blobs, xs = _cpu_sample_setup(spec)
    _cpu_token_time(ref, spec, router, blobs, xs, 1)  # warm
    n, el = 0, 0.0
    while el < budget_s and n < 256:
        el += _cpu_token_time(ref, spec, router, blobs, xs, 1)
        n += 1
    res = {"value": n / el, "unit": UNIT, "cores": ref.threads(), "kind": "reference",
           "sample": f"{n} single-token passes through one layer of the configuration via the "
                     f"reference's scalar/OpenMP CPU run_moe branch (router + shared + top-{spec.top_k} "
                     f"experts), {len(blobs)} distinct expert blobs"}
    if RefCPU.available(avx512=True):
        ra = RefCPU(avx512=True, threads=RefCPU.host_cores())
        _cpu_token_time(ra, spec, router, blobs, xs, 1)
        m = max(2, n // 2)
        t = _cpu_token_time(ra, spec, router, blobs, xs, m)
        res["avx512_build"] = {"value": m / t, "unit": UNIT, "valid_output": False,
                               "note": "reference's own -Ofast -march=icelake-server build; "
                                       "its AVX-512 int4 GEMV returns wrong values"}
    return res


def reference_arm(args, spec) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.oracle import RefCPU
    cfg = {"workload": spec.name, "layers": spec.layers, "tokens_per_step": spec.tokens,
           "hidden": spec.hidden, "inter": spec.inter, "experts": spec.n_experts,
           "shared_experts": int(spec.has_shared), "top_k": spec.top_k,
           "group_size": spec.group_size}
    line = {"impl": "reference", "metric": METRIC, "unit": UNIT, "higher_is_better": True,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "dtype": "f32", "data": "synthetic", "config": cfg, "vs_baseline": None}
    if not RefCPU.available():
        line.update({"unavailable": "reference CPU library oracle/_ref/libwisp_ref.so not built"})
        print(json.dumps(line))
        return
    # All host cores, whatever OMP_NUM_THREADS the launcher exported
    # (torch.distributed.run sets it to 1).
    ref = RefCPU(threads=RefCPU.host_cores())
    router, blobs, xs = _cpu_sample_setup(spec)
    tokens_per_step = 1
    for _ in range(args.warmup):
        _cpu_token_time(ref, spec, router, blobs, xs, tokens_per_step)
    t = _cpu_token_time(ref, spec, router, blobs, xs, tokens_per_step * args.steps)
    value = tokens_per_step * args.steps / t
    line.update({"value": value, "ms_per_step": 1e3 * t / args.steps, "scaling": "strong",
                 "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.threads(),
                                  "kind": "reference",
                                  "sample": "one token through one MoE layer per step (reference "
                                            "scalar/OpenMP CPU run_moe branch)"},
                 "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    print(json.dumps(line))


def layer_launches(T: int, world: int, has_shared: bool) -> int:
    """Our kernel launches per layer call (plus one rms_rescale between
    stacked layers, counted by the caller).

    Single GPU, T <= 4 tokens (decode chain): router logits, the decode
    planner, register-path gate/up and down = 4. Otherwise: route 2 (logits,
    top-k) + plan 2 (count and segments, ordered fill) + row pack 1 + grouped
    FFN (one tile/unit planner, register-path gate/up and down, and, when a
    segment can exceed the 32-row routing threshold, the tensor-core gate/up
    and down). Expert-parallel: route 2 + plan 2 + dispatch 2 (slots and
    entries; rows, with the rank's own rows for the shared expert) + receive
    plan + gather + one grouped FFN 5 (local experts and, over the own rows,
    the shared expert) + fp16 return rows + combine."""
    if world == 1:
        if T <= 4:
            return 4
        return 5 + (5 if T > 32 else 3)
    return 2 + 2 + 2 + 1 + 1 + 5 + 1 + 1


# ---------------------------------------------------------------------------
# The other BASELINE configurations (single GPU): one layer per step
# ---------------------------------------------------------------------------

SIDE_CONFIGS = ["mixtral_b1", "mixtral_b64", "ds_b1", "ds_b128", "ds_prefill"]


def measure_side_config(name: str, steps: int, warmup: int, peaks: dict) -> dict:
    """One MoE layer of configuration `name` (BASELINE configs[0]-[3]) as a
    step: router, dispatch, grouped FFN and combine through MoeLayer (the C
    ABI's wisp_b200_moe_forward), captured once as a CUDA graph and replayed
    (eager launches if the capture fails; reported). A single layer's touched weights (180-210
    MB at batch 1) are close to the 126 MB L2, so every step is timed alone
    with CUDA events and L2 is flushed (a 256 MB write) between steps,
    outside the timed intervals. e2e adds the host->device copy of the
    step's tokens and the device->host copy of its output."""
    import torch
    from wisp_b200 import synth
    from wisp_b200.moe import MoeLayer

    spec = synth.CONFIGS[name]
    dev = torch.device("cuda", torch.cuda.current_device())
    layers_w, x = synth.make_model(spec, dev)
    layer = MoeLayer(layers_w[0], spec.tokens)
    out = torch.empty((spec.tokens, spec.hidden), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def timed(fn, n):
        ts = []
        for _ in range(n):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.mean(ts)

    for _ in range(warmup):
        layer.forward(x, out)
    # The layer as one CUDA graph (as a serving loop replays its decode step):
    # its launches follow each other without host work between them.
    graph, graph_note = None, "on"
    try:
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            layer.forward(x, out)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            layer.forward(x, out)
        torch.cuda.synchronize()
    except Exception as exc:  # noqa: BLE001 - reported in the result
        graph, graph_note = None, f"capture failed: {type(exc).__name__}: {str(exc)[:120]}"

    def run_layer():
        if graph is not None:
            graph.replay()
        else:
            layer.forward(x, out)

    for _ in range(warmup):
        run_layer()
    ms = timed(run_layer, steps)
    layer.check()
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((spec.tokens, spec.hidden), dtype=torch.float32).pin_memory()

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        run_layer()
        out_host.copy_(out, non_blocking=True)

    e2e_step()
    ems = timed(e2e_step, steps)
    used = int(torch.unique(layer.idx).numel()) + (1 if spec.has_shared else 0)
    nbytes = used * spec.expert_bytes() + spec.n_experts * spec.hidden * 2
    R = spec.tokens * spec.top_k + (spec.tokens if spec.has_shared else 0)
    flops = 6.0 * spec.hidden * spec.inter * R + 2.0 * spec.tokens * spec.n_experts * spec.hidden
    gbs = nbytes / (ms / 1e3) / 1e9
    tfl = flops / (ms / 1e3) / 1e12
    if flops / (peaks["bf16_tflops"] * 1e12) > nbytes / (peaks["hbm_gbs"] * 1e9):
        roof = {"bound": "tensor", "achieved": round(tfl, 1), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(tfl / peaks["bf16_tflops"], 4)}
    else:
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)}
    roof.update({"kernel": "one MoE layer (router, dispatch, grouped int4 FFN, combine)",
                 "algorithmic_bytes": nbytes, "algorithmic_flops": flops,
                 "experts_touched": used, "vs_8tbs": round(gbs / 8000.0, 4),
                 "peak_source": peaks["source"], "traffic": None})
    res = {"value": round(spec.tokens / (ms / 1e3), 1), "unit": UNIT,
           "ms_per_step": round(ms, 4), "tokens_per_step": spec.tokens,
           "shape": {"hidden": spec.hidden, "inter": spec.inter, "experts": spec.n_experts,
                     "shared_experts": int(spec.has_shared), "top_k": spec.top_k,
                     "scoring": "softmax" if spec.scoring == 0 else "sigmoid group-limited",
                     "skewed_router": spec.skew},
           "l2": "flushed between steps (256 MB write, untimed)",
           "cuda_graph": graph_note,
           "roofline": roof,
           "gpu_launches": layer_launches(spec.tokens, 1, spec.has_shared) * steps,
           "e2e": {"value": round(spec.tokens / (ems / 1e3), 1), "unit": UNIT,
                   "h2d_bytes_per_step": x_host.numel() * 2,
                   "d2h_bytes_per_step": out_host.numel() * 4}}
    del graph, layer, layers_w, x, out, flush
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

PHASES = ("dispatch", "exchange", "gather", "ffn", "return", "combine")


def ep_phase_report(layers, xs, outs, step_eager, spec, T, L, world, dev, reps: int = 5) -> dict:
    """Per-phase device time of one step on every rank, and the per-rank load
    (received (token, expert) rows and touched local experts per layer).

    The step is captured as a CUDA graph with timing events recorded as graph
    nodes (external events) at the phase boundaries of every layer, then
    replayed `reps` times; phases are summed over the layers (the rms_rescale
    between layers is not counted). Falls back to eager launches if the
    capture fails."""
    import torch
    import torch.distributed as dist
    from wisp_b200 import abi
    marks = []

    def mark(name):
        ev = torch.cuda.Event(enable_timing=True, external=True)
        ev.record()
        marks.append((name, ev))

    def one_step():
        for l in range(L):
            mark("start")
            layers[l].forward(xs[l], outs[l], mark=mark)
            if l + 1 < L:
                abi.call("wisp_b200_rms_rescale", outs[l].data_ptr(), xs[l + 1].data_ptr(), T,
                         spec.hidden, 1e-6, torch.cuda.current_stream().cuda_stream)

    graph, how = None, "CUDA graph"
    try:
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_step()
        torch.cuda.synchronize()
    except Exception as exc:  # noqa: BLE001 - reported in the line
        graph, how = None, f"eager (capture failed: {type(exc).__name__})"
    ok = torch.tensor([1 if graph is not None else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok.item()) == 0 and graph is not None:
        graph.reset()
        graph, how = None, "eager (another rank failed to capture)"
    acc = {k: 0.0 for k in PHASES}
    for _ in range(reps):
        if graph is not None:
            graph.replay()
        else:
            marks.clear()
            one_step()
        torch.cuda.synchronize()
        for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
            if name != "start":
                acc[name] += a.elapsed_time(b)
    if graph is not None:
        graph.reset()   # it holds NCCL calls: released before the group
    mine = torch.tensor([acc[k] / reps for k in PHASES], dtype=torch.float64, device=dev)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    rows, touched = [], []
    for lay in layers:
        r = lay.total.to(torch.int64).reshape(1)
        seg = lay.rsegs.view(torch.int32).reshape(-1, 4)[:lay.e_loc]   # routed experts only
        u = (seg[:, 2] > 0).to(torch.int64).sum().reshape(1)
        rr = [torch.empty_like(r) for _ in range(world)]
        uu = [torch.empty_like(u) for _ in range(world)]
        dist.all_gather(rr, r)
        dist.all_gather(uu, u)
        rows.append([int(v.item()) for v in rr])
        touched.append([int(v.item()) for v in uu])
    per_rank = torch.stack(every).cpu().numpy()
    return {
        "how": f"{how} of one step with timing events between the phases of every layer, "
               f"mean of {reps} replays, summed over the {L} layers",
        "ms_per_step_max_over_ranks": {k: round(float(per_rank[:, i].max()), 4) for i, k in enumerate(PHASES)},
        "ms_per_step_rank0": {k: round(float(per_rank[0, i]), 4) for i, k in enumerate(PHASES)},
        "received_rows_per_layer": rows,
        "touched_local_experts_per_layer": touched,
    }


def ep_loopback_run(args, spec) -> None:
    """The expert-parallel layer of `args.ep_loopback` ranks run on one GPU
    (EpLayer.loopback_forward: every rank's kernels in turn, the two
    all-to-alls as block copies), for launch lists and kernel profiles of
    one rank's expert-parallel kernels without a multi-rank process. One
    JSON line: device time per loopback step of the first layer (all ranks'
    work, so not a throughput figure)."""
    import torch
    from wisp_b200 import synth
    from wisp_b200.ep import EpLayer, block_range, loopback_forward
    W = args.ep_loopback
    dev = torch.device("cuda", 0)
    one = synth.small(spec, layers=1)
    E, T = one.n_experts, one.tokens
    t_max = max(b - a for a, b in (block_range(T, W, q) for q in range(W)))
    layers, xs, outs = [], [], []
    for r in range(W):
        lw, x = synth.make_model(one, dev, keep=range(*block_range(E, W, r)))
        t0, t1 = block_range(T, W, r)
        layers.append(EpLayer(one, lw[0], t1 - t0, r, W, max_tokens=t_max))
        xs.append(x[t0:t1].contiguous())
        outs.append(torch.empty((t1 - t0, one.hidden), dtype=torch.float32, device=dev))
    for _ in range(args.warmup):
        loopback_forward(layers, xs, outs)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    a.record()
    for _ in range(args.steps):
        loopback_forward(layers, xs, outs)
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    for lay in layers:
        lay.check()
    print(json.dumps({"ep_loopback": {"ranks": W, "workload": spec.name, "layer": 0,
                                      "ms_per_loopback_step": round(a.elapsed_time(b) / args.steps, 4),
                                      "note": "every rank's kernels on one GPU, exchanges as copies"}}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="ep_stack")
    ap.add_argument("--impl", default="wisp", choices=["wisp", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step eagerly")
    ap.add_argument("--kernel-reps", type=int, default=5)
    ap.add_argument("--ep-loopback", type=int, default=0, metavar="W",
                    help="profiling aid: run the expert-parallel layer of W ranks on one GPU "
                         "(loopback exchanges) instead of the benchmark")
    ap.add_argument("--no-side-configs", action="store_true",
                    help="skip the single-layer measurements of BASELINE configs[0]-[3]")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    from wisp_b200 import synth
    spec = synth.CONFIGS[args.config]
    if args.impl == "reference":
        reference_arm(args, spec)
        return
    if args.ep_loopback:
        ep_loopback_run(args, spec)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import ctypes as C
    from wisp_b200 import abi
    from wisp_b200.moe import MoeLayer
    from wisp_b200.ep import EpLayer, block_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lib = abi.lib()
    stream = torch.cuda.current_stream()
    T_all, L = spec.tokens, spec.layers

    # -- model ------------------------------------------------------------
    keep = None if world == 1 else range(*block_range(spec.n_experts, world, rank))
    layers_w, x_all = synth.make_model(spec, dev, keep=keep)
    t0, t1 = block_range(T_all, world, rank)
    x0 = x_all[t0:t1].contiguous()
    T = t1 - t0
    if world == 1:
        layers = [MoeLayer(lw, T) for lw in layers_w]
    else:
        t_max = max(b - a for a, b in (block_range(T_all, world, q) for q in range(world)))
        layers = [EpLayer(spec, lw, T, rank, world, max_tokens=t_max) for lw in layers_w]
    outs = [torch.empty((T, spec.hidden), dtype=torch.float32, device=dev) for _ in range(L)]
    # xs[0] is the step's input buffer: callers copy their tokens into it
    xs = [x0.clone()] + [torch.empty_like(x0) for _ in range(L - 1)]

    def step_eager():
        for l in range(L):
            layers[l].forward(xs[l], outs[l])
            if l + 1 < L:
                abi.call("wisp_b200_rms_rescale", outs[l].data_ptr(), xs[l + 1].data_ptr(), T,
                         spec.hidden, 1e-6, torch.cuda.current_stream().cuda_stream)
        return outs[-1]

    def barrier():
        if world > 1:
            dist.barrier()

    # One step as a CUDA graph: the layer calls (and, across GPUs, their NCCL
    # exchanges) replay without host work between the launches. Every rank
    # captures; if any rank fails, all run eagerly.
    graph, graph_note = None, "off (--no-graph)"
    if not args.no_graph:
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    step_eager()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step_eager()
            torch.cuda.synchronize()
            graph_note = "on"
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            graph, graph_note = None, f"capture failed: {type(exc).__name__}: {str(exc)[:120]}"
        if world > 1:
            ok = torch.tensor([1 if graph is not None else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok.item()) == 0 and graph is not None:
                graph, graph_note = None, "off (another rank failed to capture)"

    def step(x_in):
        if x_in is not xs[0]:
            xs[0].copy_(x_in, non_blocking=True)
        if graph is not None:
            graph.replay()
        else:
            step_eager()
        return outs[-1]

    for _ in range(args.warmup):
        step(xs[0])
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    # keep the GPU busy while nvidia-smi starts sampling
    t_spin = time.perf_counter()
    while time.perf_counter() - t_spin < 1.0:
        step(xs[0])
        torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    ev0.record(stream)
    for _ in range(args.steps):
        step(xs[0])
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = T_all * L / (ms / 1e3)

    # error words of the bounded waits (every kernel of the step)
    for lay in layers:
        lay.check()

    # -- expert parallelism: per-phase device times and per-rank load -------
    ep_phases = None
    if world > 1:
        ep_phases = ep_phase_report(layers, xs, outs, step_eager, spec, T, L, world, dev)

    # -- algorithmic bytes of one step (routing is identical every step) --
    used = []
    for l in range(L):
        if world == 1:
            idx = layers[l].idx
        else:
            idx = layers[l].idx
        u = torch.zeros(spec.n_experts, dtype=torch.int32, device=dev)
        u[idx.reshape(-1).long()] = 1
        if world > 1:
            dist.all_reduce(u, op=dist.ReduceOp.MAX)
        used.append(int(u.sum().item()))
    eb = spec.expert_bytes()
    router_bytes = spec.n_experts * spec.hidden * 2
    shared_reads = world if spec.has_shared else 0   # every rank reads the shared expert
    step_bytes = sum((u * eb + shared_reads * eb + world * router_bytes) for u in used)
    hbm_gbs = step_bytes / (ms / 1e3) / 1e9

    # -- dominant kernel: the grouped int4 FFN (gate/up + down), timed with
    #    CUDA events around its launches on the launching stream (N=1) ------
    peaks = _peaks()
    roofline = None
    if world == 1:
        lay = layers[0]
        cfg = lay.cfg
        V = spec.n_virtual
        R = T * spec.top_k + (T if spec.has_shared else 0)
        counts = torch.empty(V, dtype=torch.int32, device=dev)
        segs = torch.empty(16 * V, dtype=torch.uint8, device=dev)
        row_token = torch.empty(R, dtype=torch.int32, device=dev)
        row_w = torch.empty(R, dtype=torch.float32, device=dev)
        xp = torch.empty((R, spec.hidden), dtype=torch.float16, device=dev)
        h = torch.empty((R, spec.inter), dtype=torch.float16, device=dev)
        gws = torch.empty(lib.wisp_b200_grouped_workspace_bytes(C.byref(cfg), V, R),
                          dtype=torch.uint8, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.zeros((T, spec.hidden), dtype=torch.float32, device=dev)
        abi.call("wisp_b200_dispatch_plan", C.byref(cfg), lay.idx.data_ptr(), lay.wt.data_ptr(),
                 counts.data_ptr(), segs.data_ptr(), row_token.data_ptr(), row_w.data_ptr(),
                 stream.cuda_stream)
        abi.call("wisp_b200_pack_rows", x0.data_ptr(), row_token.data_ptr(), R, spec.hidden,
                 xp.data_ptr(), stream.cuda_stream)
        table = [lw.prepare() for lw in layers_w]

        def ffn_calls():
            st = torch.cuda.current_stream().cuda_stream
            for l in range(L):   # rotate the layers' weights so L2 never holds them
                abi.call("wisp_b200_grouped_ffn", C.byref(cfg), table[l].data_ptr(),
                         layers_w[l].table.data_ptr(), V, segs.data_ptr(), V, R,
                         xp.data_ptr(), h.data_ptr(), 0, row_token.data_ptr(), row_w.data_ptr(),
                         out.data_ptr(), gws.data_ptr(), gws.numel(), flag.data_ptr(), st)

        # The L calls replay as one CUDA graph (as in the timed step), so the
        # host's tensor-map set-up between calls stays out of the device time.
        kgraph = None
        if graph is not None:
            ffn_calls()
            torch.cuda.synchronize()
            kgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(kgraph):
                ffn_calls()
            torch.cuda.synchronize()
        evs = []
        for rep in range(args.kernel_reps + 1):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            if kgraph is not None:
                kgraph.replay()
            else:
                ffn_calls()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        if kgraph is not None:
            kgraph.reset()
        abi.call("wisp_b200_check_error_flag", flag.data_ptr(), stream.cuda_stream)
        kms = statistics.mean(a.elapsed_time(b) for a, b in evs[1:]) / L   # first pass = warm-up
        k_bytes = (used[0] + (1 if spec.has_shared else 0)) * eb
        k_flops = 6.0 * spec.hidden * spec.inter * R     # gate, up, down per routed row
        achieved = k_bytes / (kms / 1e3) / 1e9
        tflops = k_flops / (kms / 1e3) / 1e12
        # The bound is the resource the call needs longer on at peak: HBM for
        # decode-sized groups, the tensor cores for prefill-sized ones.
        if k_flops / (peaks["bf16_tflops"] * 1e12) > k_bytes / (peaks["hbm_gbs"] * 1e9):
            bound = {"bound": "tensor", "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4)}
        else:
            bound = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4)}
        roofline = {**bound,
                    "traffic": round(k_bytes * TRAFFIC_PER_ALGORITHMIC_BYTE),
                    "traffic_source": "ncu dram__bytes_read+write of one call on ep_profile, "
                                      "scaled by algorithmic bytes",
                    "kernel": "grouped int4 FFN (gate/up+SwiGLU, down+combine)",
                    "kernel_ms": round(kms, 4), "algorithmic_bytes": k_bytes,
                    "algorithmic_flops": k_flops, "hbm_gbs": round(achieved, 1),
                    "tflops": round(tflops, 1), "peak_source": peaks["source"],
                    "vs_8tbs": round(achieved / 8000.0, 4)}

    # -- end to end through the public API with host buffers ---------------
    e2e = None
    x_host = x0.cpu().pin_memory()
    out_host = torch.empty((T, spec.hidden), dtype=torch.float32).pin_memory()
    for _ in range(2):
        xs[0].copy_(x_host, non_blocking=True)
        step(xs[0])
        out_host.copy_(outs[-1], non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xs[0].copy_(x_host, non_blocking=True)
        step(xs[0])
        out_host.copy_(outs[-1], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ems], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e = {"value": T_all * L / (ems / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": x_host.numel() * 2 * world,
           "d2h_bytes_per_step": out_host.numel() * 4 * world}

    launches_per_step = layer_launches(T, world, spec.has_shared) * L + (L - 1)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights, fp16 MMA operands, fp32 accumulate",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": spec.name, "layers": L, "tokens_per_step": T_all,
                   "hidden": spec.hidden, "inter": spec.inter, "experts": spec.n_experts,
                   "shared_experts": int(spec.has_shared), "top_k": spec.top_k,
                   "group_size": spec.group_size, "parallelism": f"ep{world}", "cuda_graph": graph_note,
                   "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB of expert weights per step)"},
        "hbm": {"step_bytes": step_bytes, "achieved_gbs": round(hbm_gbs, 1),
                "frac_of_measured": round(hbm_gbs / peaks["hbm_gbs"], 4),
                "frac_of_8tbs": round(hbm_gbs / 8000.0, 4), "experts_touched_per_layer": used},
        "roofline": roofline, "e2e": e2e, "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
        **({"ep_phases": ep_phases} if ep_phases else {}),
    }
    if world == 1 and not args.no_side_configs and args.config == "ep_stack":
        # the stack (~35 GB) stays resident; each configuration adds a few GB
        line["configs"] = {n: measure_side_config(n, args.steps, args.warmup, peaks)
                           for n in SIDE_CONFIGS}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(spec)
    if rank == 0:
        print(json.dumps(line))
    if graph is not None:   # a graph holding NCCL calls must go before the group
        graph.reset()
        graph = None
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
