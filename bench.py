"""Benchmark: Flash-Next MoE-layer decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c1]

Workload (N = 1, default ``c2``): one qwen4_exp sparse-MoE
layer -- hidden 2048, 512 experts of intermediate 512 (Q4/G32), top-10 with
softmax renorm, one Q4/G32 shared expert with a sigmoid gate -- decoding a
ragged batch of 64 tokens whose routing follows Zipf(1.1).  A step is one
full layer: router GEMV, softmax/top-k, GPU grouping, grouped gate/up+SwiGLU,
down, slot-ordered combine + shared expert.  Inputs are seeded synthetic
tensors of those shapes and distributions (no checkpoint exists here).

Four distinct layers (4 x 1.0 GB of experts, more than the 126 MB L2) are
rotated step by step, each with its own 64-token batch, so every step streams
its weights from HBM.

``value`` = tokens/s of the whole job with inputs resident in HBM (device
time, CUDA events, max over ranks).  ``e2e`` = the same through the public
API with the batch copied from pinned host memory and the output copied back
inside the timed region.  N > 1 (torchrun) runs the layer expert-parallel:
512/N experts per GPU, router and shared expert replicated, each GPU routing
its own 64 tokens (weak scaling), dispatch and return of the per-slot outputs
by the library's kernels over NVLink peer memory; device time is the max over
ranks.  That line also carries ``configs.c3``: the 48-layer C3 stack
expert-parallel over the same ranks (batch 64 and 1 per GPU), with its own
bit-identity check.

``--workload c3|c4|c5`` print one line each for the other benchmark configs
(48-layer stack -- expert-parallel under torchrun --, 5k-token prefill, paged
attention).

``--impl reference`` times the reference-semantics CPU implementation (the
NumPy oracle port; MLX, the reference's own runtime, is not installable
here) on the host cores with a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "macqwen-releases_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "MoE-layer decode tokens/s (batch 1, 64) and HBM GB/s vs roofline at 1/2/4/8 B200"
HIDDEN, INTER, EXPERTS, TOP_K, GROUP = 2048, 512, 512, 10, 32
LAYERS = 4
# bytes of one expert's three Q4/G32 projections at 2048/512
EXPERT_BYTES = 3 * (INTER * HIDDEN // 2 + 2 * INTER * (HIDDEN // GROUP) * 2)
GATE_UP_BYTES = 2 * (INTER * HIDDEN // 2 + 2 * INTER * (HIDDEN // GROUP) * 2)
ROUTER_BYTES = EXPERTS * HIDDEN * 2
# ~40 ms at B200 clocks: covers the host enqueue of the timed steps
CUSHION_CYCLES = 80_000_000


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM traffic of the gate/up launch per expert it streams (routed + shared):
# dram__bytes_read.sum 273,532,416 B (ncu, this workload's layer: 1 layer, 192
# routed experts + the shared one) + dram__bytes_write.sum 4,458,752 B (the
# full capture of the same launch), divided by 193.  Scaled to each run's
# expert count.
NCU_GATE_UP_TRAFFIC_PER_EXPERT = (273_532_416 + 4_458_752) / 193


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _max_over_ranks(value: float, world: int):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------------------
# CPU reference arm / baseline (oracle port, host cores)
# --------------------------------------------------------------------------


# The C2 layer on the host cores.  One step = the whole 64-token layer: the
# router (softmax, top-k, renorm) in the parent, the routed experts' groups
# split over spawn worker processes (the oracle's per-expert projections), the
# shared expert as one more task, then the slot-ordered combine.  Expert
# weights are generated once per process from a per-expert seed (each worker
# holds only its experts; they stay resident, as the GPU's tables do).

_CPU_STATE: dict = {}


def _cpu_layer_inputs(tokens: int, seed: int):
    """x [T,H] and router weight [E,H] (bfloat16 values as float32) with the
    C2 distributions: Zipf(1.1) expert popularity through a shared direction."""
    import numpy as np

    from oracle import bf16

    rng = np.random.default_rng(seed)
    u = rng.standard_normal(HIDDEN)
    u /= np.linalg.norm(u)
    ranks = rng.permutation(EXPERTS) + 1.0
    p = ranks ** -1.1
    p /= p.sum()
    x = bf16.round_f32((rng.standard_normal((tokens, HIDDEN)) + 8.0 * u).astype(np.float32))
    w = bf16.round_f32((rng.standard_normal((EXPERTS, HIDDEN)) * 0.02
                        + (0.43 * np.log(p) / 8.0)[:, None] * u).astype(np.float32))
    wg = bf16.round_f32((rng.standard_normal(HIDDEN) * 0.02).astype(np.float32))
    return x, w, wg


def _cpu_expert(seed: int, e: int):
    """(gate, up, down) of expert e (e = -1: the shared expert) as oracle triples."""
    import numpy as np

    from oracle import bf16

    rng = np.random.default_rng([seed, e + 1])

    def proj(o, k):
        words = rng.integers(0, 2 ** 32, (o, k // 8), dtype=np.uint32)
        sc = bf16.round_f32(np.abs(rng.normal(0, 0.01, (o, k // GROUP))).astype(np.float32))
        return words, sc, bf16.round_f32(-8 * sc)

    return proj(INTER, HIDDEN), proj(INTER, HIDDEN), proj(HIDDEN, INTER)


def _cpu_worker_init(seed: int, tokens: int):
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"
    x, _, wg = _cpu_layer_inputs(tokens, seed)
    _CPU_STATE.update(seed=seed, x=x, wg=wg, experts={})


def _cpu_task(job):
    """Worker: the per-slot down rows of its expert groups, or the shared expert."""
    import numpy as np

    from oracle import bf16, moe

    kind, payload = job
    st = _CPU_STATE
    x = st["x"]
    if kind == "shared":
        if "shared" not in st:
            st["shared"] = _cpu_expert(st["seed"], -1)
        sh, sg, sy = moe.shared_expert(x, *st["shared"], st["wg"])
        return kind, sy
    out = []
    for e, pairs in payload:
        if e not in st["experts"]:
            st["experts"][e] = _cpu_expert(st["seed"], e)
        gate, up, down = st["experts"][e]
        rows = x[np.asarray(pairs) // TOP_K]
        g = bf16.round_f32(moe.qmv(rows, moe.unpack_q4(gate[0]), gate[1], gate[2], GROUP))
        u = bf16.round_f32(moe.qmv(rows, moe.unpack_q4(up[0]), up[1], up[2], GROUP))
        act = moe.swiglu_bf16(g, u)
        d = bf16.round_f32(moe.qmv(act, moe.unpack_q4(down[0]), down[1], down[2], GROUP))
        out.append((pairs, d))
    return kind, out


class CpuLayer:
    """The C2 layer (64 tokens) on `workers` host processes; step() runs it once."""

    def __init__(self, workers: int, tokens: int = 64, seed: int = 1000):
        import multiprocessing as mp

        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = "1"  # one thread per process (inherited at spawn)
        self.tokens, self.seed, self.workers = tokens, seed, workers
        self.x, self.w, _ = _cpu_layer_inputs(tokens, seed)
        self.pool = mp.get_context("spawn").Pool(workers, initializer=_cpu_worker_init, initargs=(seed, tokens))
        self.distinct = None

    def step(self):
        import numpy as np

        from oracle import moe

        inds, scores, _, _ = moe.router(self.x, self.w, TOP_K)
        flat = inds.reshape(-1)
        experts = np.unique(flat)
        self.distinct = int(experts.size)
        groups = [(int(e), np.nonzero(flat == e)[0].tolist()) for e in experts]
        # largest groups first, dealt round-robin: balanced per-process work
        groups.sort(key=lambda g: -len(g[1]))
        jobs = [("routed", groups[i::self.workers]) for i in range(self.workers)] + [("shared", None)]
        d = np.zeros((self.tokens * TOP_K, HIDDEN), np.float32)
        sy = None
        for kind, res in self.pool.map(_cpu_task, jobs, chunksize=1):
            if kind == "shared":
                sy = res
            else:
                for pairs, rows in res:
                    d[pairs] = rows
        return moe.combine(d.reshape(self.tokens, TOP_K, HIDDEN), scores, shared_y=sy)

    def close(self):
        self.pool.terminate()
        self.pool.join()


def _cpu_workers():
    return max(1, min(os.cpu_count() or 1, 32))


def cpu_time_steps(steps: int, warmup: int, workers: int | None = None):
    """Wall time of `steps` CPU layer steps after `warmup` (each step one 64-token layer)."""
    workers = workers or _cpu_workers()
    layer = CpuLayer(workers)
    try:
        for _ in range(max(1, warmup)):  # the first step also generates each worker's experts
            layer.step()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            layer.step()
            times.append(time.perf_counter() - t0)
    finally:
        layer.close()
    return times, layer.distinct, workers


def cpu_baseline(steps: int = 4):
    """The C2 layer on all host cores; returns (tokens/s, sample, cores)."""
    times, distinct, workers = cpu_time_steps(steps, 1)
    rate = 64 * len(times) / sum(times)
    sample = (f"{len(times)} steps of the 64-token C2 layer (router in the parent; {distinct} distinct experts "
              f"split over {workers} spawn processes + the shared expert; median "
              f"{1000 * statistics.median(times):.0f} ms/step)")
    return rate, sample, workers


def reference_arm(args):
    world, rank, _ = _dist()
    if rank != 0:
        return 0
    times, distinct, workers = cpu_time_steps(args.steps, args.warmup)
    total = sum(times)
    value = 64 * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "C2: one qwen4_exp MoE layer, 64-token ragged decode, Zipf(1.1) routing, "
                               "H2048/I512/E512 top-10 Q4/G32 + Q4/G32 shared expert",
                   "tokens_per_gpu": 64, "distinct_experts_per_layer": distinct},
        "step_ms": {"median": 1000 * statistics.median(times), "p10": 1000 * _pct(times, 10),
                    "p90": 1000 * _pct(times, 90)},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": workers, "kind": "port",
                         "sample": f"{len(times)} steps, each the whole 64-token layer: router in the parent, "
                                   f"{distinct} expert groups over {workers} spawn processes + the shared expert"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "NumPy restatement of the reference semantics on host cores (the MLX runtime of the "
                "reference is not installable here)",
    }
    print(json.dumps(line), flush=True)
    return 0


def _pct(values, q):
    """q-th percentile (linear interpolation) of a list of numbers."""
    v = sorted(values)
    if not v:
        return None
    pos = (len(v) - 1) * q / 100.0
    lo = int(pos)
    hi = min(lo + 1, len(v) - 1)
    return v[lo] + (v[hi] - v[lo]) * (pos - lo)


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------


def _build_layers(tokens, layers, seed):
    from flashnext_b200 import synthetic
    from flashnext_b200.moe_block import SparseMoEBlock

    blocks, xs = [], []
    for i in range(layers):
        L = synthetic.moe_layer(tokens, HIDDEN, INTER, EXPERTS, TOP_K, GROUP, zipf=1.1, seed=seed + 101 * i)
        blocks.append(SparseMoEBlock(L.router_weight, L.experts, top_k=TOP_K, shared=L.shared,
                                     shared_expert_gate=L.shared_expert_gate))
        xs.append(L.x)
    return blocks, xs


def _distinct_experts(block):
    import torch

    return int(torch.unique(block.last_inds).numel())


def gpu_arm(args):
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from flashnext_b200 import _lib

    _lib.ensure_device()
    tokens = 64 if args.workload == "c2" else 1
    layers = max(1, args.layers)
    blocks, xs = _build_layers(tokens, layers, seed=17 + rank)
    outs = [torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device="cuda") for _ in range(layers)]
    stream = torch.cuda.current_stream()

    def step(i):
        j = i % layers
        blocks[j](xs[j], out=outs[j])

    warm = max(3, args.warmup, layers)
    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    used = [(_distinct_experts(b)) for b in blocks]

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # A spin kernel ahead of the start event keeps the device busy while the
    # host enqueues the timed steps, so the events bracket device work only.
    torch.cuda._sleep(CUSHION_CYCLES)
    start.record(stream)
    for i in range(args.steps):
        step(i)
    end.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    ms = start.elapsed_time(end)
    clocks = sampler.stop()
    ms = _max_over_ranks(ms, world)
    value = tokens * args.steps * world / (ms / 1000.0)

    # e2e: pinned host batch -> device -> layer -> host, per step
    host_x = [x.cpu().pin_memory() for x in xs]
    host_out = [torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory() for _ in range(layers)]
    dev_x = [torch.empty_like(x) for x in xs]

    def e2e_step(i):
        j = i % layers
        dev_x[j].copy_(host_x[j], non_blocking=True)
        blocks[j](dev_x[j], out=outs[j])
        host_out[j].copy_(outs[j], non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_serial_ms = _max_over_ranks(e0.elapsed_time(e1), world)

    # The same steps as a serving loop runs them: step i's input copy (copy
    # stream) and its output read (second copy stream) overlap the layers of
    # the neighbouring steps; every copy is still inside the timed region.
    # Buffer j is reused every `layers` steps, after the step that last used
    # it is done with it.
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()
    x_ready = [torch.cuda.Event() for _ in range(layers)]
    y_ready = [torch.cuda.Event() for _ in range(layers)]
    x_free = [torch.cuda.Event() for _ in range(layers)]
    y_free = [torch.cuda.Event() for _ in range(layers)]
    for j in range(layers):
        x_free[j].record(stream)
        y_free[j].record(stream)

    def e2e_overlapped(n):
        for i in range(n):
            j = i % layers
            with torch.cuda.stream(h2d_s):
                h2d_s.wait_event(x_free[j])
                dev_x[j].copy_(host_x[j], non_blocking=True)
                x_ready[j].record(h2d_s)
            stream.wait_event(x_ready[j])
            stream.wait_event(y_free[j])
            blocks[j](dev_x[j], out=outs[j])
            x_free[j].record(stream)
            y_ready[j].record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(y_ready[j])
                host_out[j].copy_(outs[j], non_blocking=True)
                y_free[j].record(d2h_s)
        for s_ in (h2d_s, d2h_s):
            stream.wait_stream(s_)

    e2e_overlapped(3)
    torch.cuda.synchronize()
    _barrier(world)
    e0.record(stream)
    h2d_s.wait_event(e0)
    d2h_s.wait_event(e0)
    e2e_overlapped(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = tokens * args.steps * world / (e2e_ms / 1000.0)
    e2e_serial_value = tokens * args.steps * world / (e2e_serial_ms / 1000.0)

    # per-kernel device times (separate pass of the same steps, events per launch)
    _lib.profile_enable(True)
    _lib.profile_read(reset=True)
    torch.cuda._sleep(CUSHION_CYCLES)
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    prof = _lib.profile_read(reset=True)
    _lib.profile_enable(False)
    launches_per_step = sum(c for c, _ in prof.values()) / max(1, args.steps)

    hbm_peak, peak_kind = _peaks()
    avg_used = sum(used) / len(used)
    gu_count, gu_ms = prof.get("gate_up", (0, 0.0))
    gu_avg_s = (gu_ms / max(1, gu_count)) / 1000.0
    gu_bytes = (avg_used + 1) * GATE_UP_BYTES + tokens * HIDDEN * 2 * (TOP_K + 1)
    achieved = gu_bytes / gu_avg_s / 1e9 if gu_avg_s > 0 else None
    layer_bytes = (avg_used + 1) * EXPERT_BYTES + ROUTER_BYTES + HIDDEN * 2 + 2 * tokens * HIDDEN * 2
    step_s = ms / args.steps / 1000.0

    # per-step distribution over 200 more steps (events between steps)
    distribution = step_distribution(step, 200) if world == 1 else None

    batch1 = None
    if world == 1 and args.workload == "c2" and not args.no_batch1:
        batch1 = batch1_numbers(hbm_peak)

    # the other benchmark configs, one GPU (weights of each config are freed before the next)
    configs = {}
    if world == 1 and args.workload == "c2" and not args.no_configs:
        del blocks, xs, outs, host_x, host_out, dev_x
        torch.cuda.empty_cache()
        configs["c5"] = c5_numbers(20, 3)
        configs["c4"] = c4_numbers(5, 3)
        configs["c3"] = c3_numbers(10)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, sample, cores = cpu_baseline()
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": "C2: one qwen4_exp MoE layer, 64-token ragged decode, Zipf(1.1) routing, "
                            "H2048/I512/E512 top-10 Q4/G32 + Q4/G32 shared expert" if tokens == 64 else
                            "C1: one MoE layer, batch-1 decode",
                "tokens_per_gpu": tokens, "layers_rotated": layers,
                "l2": f"inputs larger than L2: {layers} distinct 1.0 GB layers rotated per step",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "distinct_experts_per_layer": avg_used,
            },
            "layer_hbm_gbs": layer_bytes / step_s / 1e9,
            "layer_roofline_frac": (layer_bytes / step_s / 1e9) / hbm_peak,
            "roofline": {"bound": "hbm", "kernel": "gate_up", "achieved": achieved, "peak": hbm_peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": (achieved / hbm_peak) if achieved else None,
                         "traffic": NCU_GATE_UP_TRAFFIC_PER_EXPERT * (avg_used + 1),
                         "algorithmic_bytes": gu_bytes, "avg_launch_us": gu_avg_s * 1e6},
            "kernels": {k: {"launches": c, "avg_us": 1000.0 * t / max(1, c)} for k, (c, t) in prof.items()},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": tokens * HIDDEN * 2,
                    "d2h_bytes_per_step": tokens * HIDDEN * 2,
                    "copies": "pinned host -> device input and device -> pinned host output of every step "
                              "inside the timed region, on two copy streams overlapping the neighbouring "
                              "steps' layers",
                    "serialized_value": e2e_serial_value},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if distribution is not None:
            line["step_ms"] = distribution
        if batch1 is not None:
            line["batch1"] = batch1
        if configs:
            line["configs"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def ep_arm(args):
    """N > 1: the C2 layer expert-parallel over N GPUs (experts 512/N per rank,
    router and shared expert replicated, 64 tokens routed by each rank;
    dispatch of the x rows and return of the per-slot outputs by the
    library's own kernels over NVLink peer memory, ``fnmoe_ep_*``; NCCL only
    for set-up and the parity check)."""
    import datetime

    import torch
    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.expert_parallel import CudaBackend, ExpertParallelMoE

    _lib.ensure_device()
    from flashnext_b200.moe_block import SparseMoEBlock

    tokens = 64
    layers = max(1, args.layers)
    per = EXPERTS // world
    eps, xs = [], []
    ref_block = None
    for i in range(layers):
        L = synthetic.moe_layer(tokens * world, HIDDEN, INTER, EXPERTS, TOP_K, GROUP, zipf=1.1, seed=17 + 101 * i)
        local_bank = {n: tuple(t[rank * per:(rank + 1) * per].contiguous() for t in v) for n, v in L.experts.items()}
        backend = CudaBackend(L.router_weight, local_bank, L.shared, L.shared_expert_gate, top_k=TOP_K)
        eps.append(ExpertParallelMoE(backend, expert_count=EXPERTS, hidden_size=HIDDEN, top_k=TOP_K,
                                     capacity_tokens=tokens))
        xs.append(L.x[tokens * rank:tokens * (rank + 1)].contiguous())
        if i == 0:  # the whole layer on this GPU: the bit-identity reference
            ref_block = SparseMoEBlock(L.router_weight, L.experts, top_k=TOP_K, shared=L.shared,
                                       shared_expert_gate=L.shared_expert_gate)
        del L, local_bank
    torch.cuda.synchronize()
    # parity: layer 0 expert-parallel vs all 512 experts on one GPU, bit for bit, every rank
    same = torch.equal(eps[0](xs[0]).view(torch.int16), ref_block(xs[0]).view(torch.int16))
    flag = torch.tensor([1 if same else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    parity = bool(flag.item())
    del ref_block
    torch.cuda.empty_cache()

    def eager_step(i):
        j = i % layers
        return eps[j](xs[j])

    warm = max(3, args.warmup, layers)
    for i in range(warm):
        eager_step(i)
    torch.cuda.synchronize()
    # One CUDA graph per layer (the peer-memory exchange kernels included:
    # with a fixed capacity the step reads nothing back to the host).  Every rank must
    # agree that capture worked before any graph is replayed.
    graphs, gouts = [], []  # the only references to the graphs: cleared before the process group goes
    ok = 1
    try:
        _capture_ep_graphs(eps, xs, graphs, gouts)
    except Exception as exc:  # fall back to eager steps on every rank
        print(f"rank {rank}: graph capture failed: {exc!r}", file=sys.stderr, flush=True)
        ok = 0
    flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    use_graphs = bool(flag.item())
    if not use_graphs:
        graphs.clear()
        gouts.clear()

    def step(i):
        if use_graphs:
            graphs[i % layers].replay()
            return gouts[i % layers]
        return eager_step(i)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(CUSHION_CYCLES)
    start.record(stream)
    for i in range(args.steps):
        step(i)
    end.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    ms = _max_over_ranks(start.elapsed_time(end), world)
    clocks = sampler.stop()
    value = tokens * args.steps * world / (ms / 1000.0)

    host_x = [x.cpu().pin_memory() for x in xs]
    host_out = [torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory() for _ in range(layers)]
    dev_x = [torch.empty_like(x) for x in xs]

    def e2e_step(i):
        # the batch lands in the step's input buffer (the graph's input), the output goes back to the host
        j = i % layers
        xs[j].copy_(host_x[j], non_blocking=True)
        host_out[j].copy_(step(j), non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = tokens * args.steps * world / (e2e_ms / 1000.0)

    _lib.profile_enable(True)
    _lib.profile_read(reset=True)
    for i in range(args.steps):
        eager_step(i)
    torch.cuda.synchronize()
    prof = _lib.profile_read(reset=True)
    _lib.profile_enable(False)
    _barrier(world)
    launches_per_step = sum(c for c, _ in prof.values()) / max(1, args.steps)
    hbm_peak, peak_kind = _peaks()
    gu_count, gu_ms = prof.get("gate_up", (0, 0.0))
    gu_avg_s = (gu_ms / max(1, gu_count)) / 1000.0

    def avg_us(name):
        c, t = prof.get(name, (0, 0.0))
        return 1000.0 * t / max(1, c)

    exchange_us = {"dispatch": avg_us("ep_dispatch"), "return_combine": avg_us("ep_return_combine")}
    # the 48-layer C3 stack expert-parallel over the same ranks (collective)
    c3 = None if args.no_configs else c3_ep_numbers(10)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "parity_vs_1gpu": parity,
            "exchange_us": exchange_us,
            "config": {"workload": "C2 layer, expert-parallel: 64 Zipf(1.1)-routed tokens per GPU, "
                                   f"512 experts sharded {per}/GPU, router + shared expert replicated",
                       "tokens_per_gpu": tokens, "layers_rotated": layers,
                       "l2": f"inputs larger than L2: {layers} distinct layers rotated per step",
                       "parallelism": f"ep{world}", "cuda_graph": use_graphs,
                       "exchange": "NVLink peer stores into CUDA-IPC windows: one row per (token, owner rank), "
                                   "per-slot outputs returned exact-size, epoch flags (no collective library)",
                       "parity": "layer 0, every rank: bit-identical to all 512 experts on one GPU"},
            "roofline": {"bound": "hbm", "kernel": "gate_up", "avg_launch_us": gu_avg_s * 1e6,
                         "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s", "achieved": None,
                         "frac": None, "traffic": None,
                         "note": "per-rank expert kernels; see the single-GPU line for the roofline"},
            "kernels": {k: {"launches": c, "avg_us": 1000.0 * t / max(1, c)} for k, (c, t) in prof.items()},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": tokens * HIDDEN * 2,
                    "d2h_bytes_per_step": tokens * HIDDEN * 2},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "clocks": clocks, "cpu_baseline": None,
        }
        if c3 is not None:
            line["configs"] = {"c3": c3}
        print(json.dumps(line), flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    graphs.clear()  # graphs go before the exchange windows and the process group
    gouts.clear()
    import gc

    gc.collect()
    torch.cuda.synchronize()
    for ep in eps:
        ep.close()
    dist.destroy_process_group()
    return 0


def _capture_ep_graphs(eps, xs, graphs, gouts):
    """One CUDA graph per expert-parallel layer step (appended to `graphs`,
    outputs to `gouts`); no other reference to a graph outlives this call."""
    import torch

    cap_stream = torch.cuda.Stream()
    cap_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap_stream):
        for ep, x in zip(eps, xs):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], stream=cap_stream):
                gouts.append(ep(x))
    torch.cuda.current_stream().wait_stream(cap_stream)
    torch.cuda.synchronize()


def step_distribution(step, n):
    """Device time of each of n more steps (CUDA events between the steps,
    after a spin kernel that covers the host enqueue): median, p10, p90 (ms)."""
    import torch

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
    torch.cuda.synchronize()
    torch.cuda._sleep(CUSHION_CYCLES)
    ev[0].record()
    for i in range(n):
        step(i)
        ev[i + 1].record()
    torch.cuda.synchronize()
    ts = [ev[i].elapsed_time(ev[i + 1]) for i in range(n)]
    return {"steps": n, "median_ms": statistics.median(ts), "p10_ms": _pct(ts, 10), "p90_ms": _pct(ts, 90)}


def batch1_numbers(hbm_peak):
    """Batch-1 (config 1) tokens/s over 8 distinct layers via one CUDA graph."""
    import torch

    layers = 8
    blocks, xs = _build_layers(1, layers, seed=900)
    outs = [torch.empty((1, HIDDEN), dtype=torch.bfloat16, device="cuda") for _ in range(layers)]
    for j in range(layers):
        blocks[j](xs[j], out=outs[j])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for j in range(layers):
                blocks[j](xs[j], out=outs[j])
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = 20
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (reps * layers)
    layer_bytes = (TOP_K + 1) * EXPERT_BYTES + ROUTER_BYTES + HIDDEN * 2 * 3
    gbs = layer_bytes / (ms / 1000.0) / 1e9
    return {"layer_tokens_per_s": 1000.0 / ms, "us_per_layer": ms * 1000.0, "hbm_gbs": gbs,
            "roofline_frac": gbs / hbm_peak, "bytes_per_layer": layer_bytes,
            "note": "8 distinct layers in one CUDA graph, 20 replays"}


# --------------------------------------------------------------------------
# Other benchmark configs (one JSON line each; the default line is C2)
# --------------------------------------------------------------------------


def _timed(fn, steps, cushion=True):
    """Device time (ms) of `steps` calls of fn(i), events on the current stream."""
    import torch

    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if cushion:
        torch.cuda._sleep(CUSHION_CYCLES)
    a.record()
    for i in range(steps):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def _graph(fn):
    """Capture fn() into a CUDA graph (after one eager call)."""
    import torch

    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    return g


def c5_numbers(steps: int, warmup: int) -> dict:
    """Config 5: paged-KV decode attention, GQA 16/2, D 256, page 64, 16 sequences
    with context ~ U[1k, 32k]; two KV pools (each > L2) alternate per step."""
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.paged_attention import paged_decode

    _lib.ensure_device()
    hbm_peak, peak_kind = _peaks()
    sets = [synthetic.paged_decode_inputs(16, 16, 2, 256, 64, (1024, 32768), seed=500 + i) for i in range(2)]
    outs = [torch.empty_like(P.q) for P in sets]

    def step(i):
        P = sets[i % 2]
        paged_decode(P.q, P.k_cache, P.v_cache, P.block_table, P.context_lens, P.scale, out=outs[i % 2])

    for i in range(max(3, warmup)):
        step(i)
    ms = _timed(step, steps) / steps
    ctx = [int(P.context_lens.sum()) for P in sets]
    kv_bytes = sum(ctx) / 2 * 2048  # K and V, 2 KV heads x 256 x 2 B per context token (mean of the two sets)
    io = 2 * 16 * 16 * 256 * 2
    gbs = (kv_bytes + io) / (ms / 1000.0) / 1e9
    del sets, outs
    torch.cuda.empty_cache()
    return {
        "metric": "paged-KV decode attention GB/s (C5)", "value": gbs, "unit": "GB/s", "steps": steps,
        "ms_per_step": ms, "workload": "C5: 16 sequences, GQA 16/2, head_dim 256, page 64, ctx U[1k,32k]",
        "context_tokens": ctx, "l2": "two KV pools of ~0.5 GB alternate",
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": gbs / hbm_peak},
    }


def c5_arm(args):
    r = c5_numbers(args.steps, args.warmup)
    print(json.dumps({
        "metric": r["metric"], "value": r["value"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": r["ms_per_step"], "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": r["workload"], "context_tokens": r["context_tokens"],
                                        "l2": r["l2"]},
        "roofline": r["roofline"],
    }), flush=True)
    return 0


def c3_numbers(steps: int) -> dict:
    """Config 3: 48-layer stack, hidden 3072, 512 experts of intermediate 640 +
    shared, top-10, Q4/G32; batch-1 and batch-64 decode through all 48 layers
    (CUDA graph replays).  Each layer is generated, tiled and its arrays freed
    before the next, so ~97 GB of tiled experts stay resident."""
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock

    _lib.ensure_device()
    hbm_peak, peak_kind = _peaks()
    H, I, E, K, n_layers = 3072, 640, 512, 10, 48
    blocks, routers = [], []
    for l in range(n_layers):
        L = synthetic.moe_layer(64, H, I, E, K, 32, zipf=1.1, seed=7000 + 31 * l)
        blocks.append(SparseMoEBlock(L.router_weight, L.experts, top_k=K, shared=L.shared,
                                     shared_expert_gate=L.shared_expert_gate))
        routers.append(L.x)
        del L
        torch.cuda.synchronize()
    expert_bytes = 3 * (I * H // 2 + 2 * I * (H // 32) * 2)
    results = {}
    for tokens in (1, 64):
        xs = [routers[l][:tokens].contiguous() for l in range(n_layers)]
        outs = [torch.empty((tokens, H), dtype=torch.bfloat16, device="cuda") for _ in range(n_layers)]

        def stack():
            for l in range(n_layers):
                blocks[l](xs[l], out=outs[l])

        g = _graph(stack)
        for _ in range(3):
            g.replay()
        ms = _timed(lambda i: g.replay(), steps) / steps
        used = [int(torch.unique(b.last_inds).numel()) for b in blocks]
        step_bytes = sum((u + 1) * expert_bytes for u in used) + n_layers * (E * H * 2 + H * 2)
        gbs = step_bytes / (ms / 1000.0) / 1e9
        results[f"batch{tokens}"] = {"tokens_per_s": tokens / (ms / 1000.0), "ms_per_token_step": ms,
                                     "hbm_gbs": gbs, "roofline_frac": gbs / hbm_peak,
                                     "distinct_experts_per_layer": sum(used) / len(used)}
        del g
    resident = sum(b.tiled.gate_up.numel() + b.tiled.down.numel() for b in blocks) / 1e9
    del blocks, routers
    torch.cuda.empty_cache()
    return {"metric": "48-layer MoE decode tokens/s (C3)", "value": results["batch64"]["tokens_per_s"],
            "unit": "tokens/s", "steps": steps,
            "workload": "C3: 48 layers, H3072/I640/E512 top-10 Q4/G32 + shared, Zipf(1.1) routing; "
                        "value = batch-64 tokens/s, batch1 below",
            "resident_tiled_gb": resident, "results": results, "peak": hbm_peak, "peak_kind": peak_kind}


def c3_arm(args):
    r = c3_numbers(args.steps)
    print(json.dumps({
        "metric": r["metric"], "value": r["value"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": 3, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": r["workload"], "resident_tiled_gb": r["resident_tiled_gb"]},
        "results": r["results"], "peak": r["peak"], "peak_kind": r["peak_kind"],
    }), flush=True)
    return 0


def c3_ep_numbers(steps: int) -> dict:
    """Config 3 expert-parallel over the ranks of the initialised process
    group: the 48-layer stack, H3072/I640/E512 top-10 Q4/G32 + shared,
    512/N experts of every layer per rank (tiled), router and shared expert
    replicated, the library's NVLink peer-memory exchange in every layer.
    Each rank routes its own batch (64 tokens, then 1: weak scaling); one CUDA
    graph per layer, the 48 replayed in order per step; device time max over
    ranks.  Layer 0 is checked bit for bit against all 512 experts on one
    GPU, on every rank.  Collective: every rank calls it."""
    import gc

    import torch
    import torch.distributed as dist

    from flashnext_b200 import synthetic
    from flashnext_b200.expert_parallel import CudaBackend, ExpertParallelMoE
    from flashnext_b200.moe_block import SparseMoEBlock

    world, rank, _ = _dist()
    H, I, E, K, n_layers, cap = 3072, 640, 512, 10, 48, 64
    per = E // world
    eps, xs = [], []
    parity = False
    for l in range(n_layers):
        L = synthetic.moe_layer(cap * world, H, I, E, K, 32, zipf=1.1, seed=7000 + 31 * l)
        local_bank = {n: tuple(t[rank * per:(rank + 1) * per].contiguous() for t in v) for n, v in L.experts.items()}
        backend = CudaBackend(L.router_weight, local_bank, L.shared, L.shared_expert_gate, top_k=K)
        eps.append(ExpertParallelMoE(backend, expert_count=E, hidden_size=H, top_k=K, capacity_tokens=cap))
        xs.append(L.x[cap * rank:cap * (rank + 1)].contiguous())
        if l == 0:  # every rank takes this collective step at the same point
            ref = SparseMoEBlock(L.router_weight, L.experts, top_k=K, shared=L.shared,
                                 shared_expert_gate=L.shared_expert_gate)
            parity = torch.equal(eps[0](xs[0]).view(torch.int16), ref(xs[0]).view(torch.int16))
            del ref
        del L, local_bank, backend
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    flag = torch.tensor([1 if parity else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    parity = bool(flag.item())
    stream = torch.cuda.current_stream()
    results = {}
    for batch in (64, 1):
        bx = [x[:batch].contiguous() for x in xs]
        for ep, x in zip(eps, bx):  # eager warm-up of every layer at this batch
            ep(x)
        torch.cuda.synchronize()
        graphs, gouts = [], []
        _capture_ep_graphs(eps, bx, graphs, gouts)
        for _ in range(3):
            for g in graphs:
                g.replay()
        torch.cuda.synchronize()
        _barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(CUSHION_CYCLES)
        start.record(stream)
        for _ in range(steps):
            for g in graphs:
                g.replay()
        end.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        ms = _max_over_ranks(start.elapsed_time(end), world) / steps
        results[f"batch{batch}"] = {"tokens_per_s": batch * world / (ms / 1000.0), "ms_per_token_step": ms,
                                    "tokens_per_gpu": batch}
        graphs.clear()  # the graphs go before the exchange windows and the process group
        gouts.clear()
        gc.collect()
        torch.cuda.synchronize()
    for ep in eps:
        ep.close()
    del eps, xs
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"metric": "48-layer MoE decode tokens/s (C3)", "value": results["batch64"]["tokens_per_s"],
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "scaling": "weak", "parity_vs_1gpu": parity,
            "workload": "C3: 48 layers, H3072/I640/E512 top-10 Q4/G32 + shared, Zipf(1.1) routing, "
                        f"experts sharded {per}/GPU, router + shared expert replicated; value = batch-64-per-GPU "
                        "tokens/s of the whole job, batch1 below",
            "parallelism": f"ep{world}", "results": results}


def c3_ep_arm(args):
    """``--workload c3`` under torchrun (N > 1): the expert-parallel 48-layer
    stack as its own line (c3_ep_numbers)."""
    import datetime

    import torch
    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from flashnext_b200 import _lib

    _lib.ensure_device()
    hbm_peak, peak_kind = _peaks()
    r = c3_ep_numbers(args.steps)
    if rank == 0:
        print(json.dumps({
            "metric": r["metric"], "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": 3, "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
            "parity_vs_1gpu": r["parity_vs_1gpu"],
            "config": {"workload": r["workload"], "parallelism": r["parallelism"], "cuda_graph": True,
                       "exchange": "NVLink peer stores into CUDA-IPC windows (the library's kernels)",
                       "parity": "layer 0, every rank: bit-identical to all 512 experts on one GPU"},
            "results": r["results"], "peak": hbm_peak, "peak_kind": peak_kind,
        }), flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    dist.destroy_process_group()
    return 0


def c4_numbers(steps_arg: int, warmup: int) -> dict:
    """Config 4: 5,000-token prefill chunk through one H2048/I512/E512 top-10
    Q4/G32 layer (+ shared), uniform routing.  The layer picks the tcgen05
    grouped GEMMs (prefill path); value = TFLOP/s of the expert GEMMs
    (routed 2*50,000*3*2048*512 + shared 2*5,000*3*2048*512 + router) over
    the layer time.  The roofline is the gate/up GEMM kernel's useful FLOPs
    over its own event-timed launches; the exact decode-path kernels on the
    same layer are reported beside it."""
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock

    _lib.ensure_device()
    tokens = 5000
    L = synthetic.moe_layer(tokens, HIDDEN, INTER, EXPERTS, TOP_K, GROUP, zipf=None, seed=4242)
    kw = dict(top_k=TOP_K, shared=L.shared, shared_expert_gate=L.shared_expert_gate)
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device="cuda")
    pairs = tokens * (TOP_K + 1)
    flops = 2.0 * pairs * 3 * HIDDEN * INTER + 2.0 * tokens * (EXPERTS + 1) * HIDDEN
    gu_flops = 2.0 * pairs * 2 * INTER * HIDDEN
    dn_flops = 2.0 * pairs * INTER * HIDDEN
    d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(d.get("bf16_tflops", 1590.0))
    peak_kind = "measured burst" if "bf16_tflops" in d else "fallback"
    steps = max(1, min(steps_arg, 10))
    res = {}
    for path in ("prefill", "decode"):
        block = SparseMoEBlock(L.router_weight, L.experts, path=path, **kw)
        for _ in range(max(3, warmup)):
            block(L.x, out=out)
        ms = _timed(lambda i: block(L.x, out=out), steps) / steps
        _lib.profile_enable(True)
        _lib.profile_read(reset=True)
        torch.cuda._sleep(CUSHION_CYCLES)
        for _ in range(steps):
            block(L.x, out=out)
        torch.cuda.synchronize()
        prof = _lib.profile_read(reset=True)
        _lib.profile_enable(False)
        kern = {k: {"launches": c, "avg_us": 1000.0 * t / max(1, c)} for k, (c, t) in prof.items()}
        res[path] = {"ms_per_step": ms, "tflops": flops / (ms / 1000.0) / 1e12, "kernels": kern}
        del block
        torch.cuda.empty_cache()
    pk = res["prefill"]["kernels"]
    gu_us = pk.get("gate_up", {}).get("avg_us", 0.0)
    dn_us = pk.get("down", {}).get("avg_us", 0.0)
    gu_tf = gu_flops / (gu_us * 1e-6) / 1e12 if gu_us else None
    ms = res["prefill"]["ms_per_step"]
    tflops = res["prefill"]["tflops"]
    del L
    torch.cuda.empty_cache()
    return {"metric": "prefill MoE layer TFLOP/s (C4)", "value": tflops, "unit": "TFLOP/s", "steps": steps,
            "ms_per_step": ms,
            "workload": "C4: 5,000 tokens, H2048/I512/E512 top-10 Q4/G32 + shared, uniform routing",
            "kernel": "tcgen05 grouped GEMM (M128 N256 K16 bf16, fp32 TMEM accumulators), "
                      "Q4 dequant to bf16 in registers",
            "roofline": {"bound": "tensor", "kernel": "prefill gate_up", "achieved": gu_tf, "peak": peak,
                         "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": (gu_tf / peak) if gu_tf else None,
                         "useful_flops": gu_flops, "avg_launch_us": gu_us},
            "down_tflops": dn_flops / (dn_us * 1e-6) / 1e12 if dn_us else None, "paths": res}


def c4_arm(args):
    r = c4_numbers(args.steps, args.warmup)
    print(json.dumps({
        "metric": r["metric"], "value": r["value"], "unit": "TFLOP/s", "n_gpus": 1, "steps": r["steps"],
        "warmup": max(3, args.warmup), "ms_per_step": r["ms_per_step"], "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": r["workload"], "kernel": r["kernel"]},
        "roofline": r["roofline"], "down_tflops": r["down_tflops"], "paths": r["paths"],
    }), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c1", "c3", "c4", "c5"], default="c2",
                    help="c2 (default) is the headline line; c3/c4/c5 print their own lines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS, help="distinct layers rotated per step")
    ap.add_argument("--no-batch1", action="store_true", help="skip the batch-1 CUDA-graph sub-measure")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the C3/C4/C5 sub-measures of the default line (one GPU), "
                         "or its expert-parallel C3 sub-measure (N > 1)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "c5":
        return c5_arm(args)
    if args.workload == "c3":
        return c3_ep_arm(args) if _dist()[0] > 1 else c3_arm(args)
    if args.workload == "c4":
        return c4_arm(args)
    if _dist()[0] > 1:
        return ep_arm(args)
    return gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
