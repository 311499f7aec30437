"""Benchmark of the Q4 quantized-linear hot path on B200.

Default workload: the seven Q4_0 linears of one
Llama-2-7B layer (Q, K, V, O: 4096->4096; gate, up: 4096->11008; down:
11008->4096) at decode batch 1, 4 and 16 -- a "step" is one pass over all
3 x 7 GEMVs, issued the way the engine issues them (QKV as one multi call,
O, gate/up as one multi call, down; swamp-engine/src/executor.rs:439-505).
Weights are random-init GGUF Q4_0 blocks from a fixed seed; >= 5 distinct
copies of the layer rotate so every GEMV streams from HBM (the rotation
footprint exceeds 4x the 126 MB L2).

metric: whole-job algorithmic GB/s (weights N*K*18/32 bytes + activations in
+ outputs out). With --gpus N (torchrun, one rank
per GPU) the model has N such layers, each tensor-parallel over the N ranks
(column split Q/K/V/gate/up, row split O/down + NCCL all-reduce), so per-GPU
bytes stay fixed (weak scaling).

--impl reference times the reference's CPU path (the C restatement of
swamp-engine forward_linear: per call, full-tensor dequant + f32 row dots,
row-partitioned over host threads) on a bounded sample of the same workload.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llamanyon.rs_b200"))

SEED = 0x5EED1A11
Q40, Q4K = 2, 12
# (name, K, N) of one Llama-2-7B layer
LAYER = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
         ("gate", 4096, 11008), ("up", 4096, 11008), ("down", 11008, 4096)]
TP_MODE = {"q": 1, "k": 1, "v": 1, "gate": 1, "up": 1, "o": 2, "down": 2}
BATCHES = (1, 4, 16)
METRIC = "Q4_0 decode GEMV GB/s (Llama-2-7B layer linears, batch 1/4/16)"


def wbytes(k, n):
    return n * k * 18 // 32


def step_bytes(n_layers=1):
    """algorithmic bytes of one step (114,148,352 /
    115,085,312 / 118,833,152 per layer at batch 1/4/16)."""
    tot = 0
    for b in BATCHES:
        for _, k, n in LAYER:
            tot += wbytes(k, n) + b * (k + n) * 4
    return tot * n_layers


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------

def cpu_sample(threads, seconds_budget=20.0, max_calls=None):
    """The reference CPU path on the layer at batch 1 (one token), repeated
    while inside the time budget. Returns (GB/s, calls, seconds, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import numpy as np
    oracle.build()
    ws = [(k, n, oracle.gen_weight(Q40, SEED, 500 + i, n, k)) for i, (_, k, n) in enumerate(LAYER)]
    x = {k: oracle.gen_x(SEED, 900 + k, (k,)) for _, k, _ in LAYER}
    # one warm call (page-in)
    oracle.forward_linear(Q40, ws[0][2], x[ws[0][0]], ws[0][1], ws[0][0], threads)
    t0 = time.perf_counter()
    calls, nbytes = 0, 0
    while True:
        for k, n, w in ws:
            oracle.forward_linear(Q40, w, x[k], n, k, threads)
            calls += 1
            nbytes += wbytes(k, n) + (k + n) * 4
        el = time.perf_counter() - t0
        if el > seconds_budget or (max_calls and calls >= max_calls):
            break
    return nbytes / el / 1e9, calls, el


def reference_arm(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    per_step = []
    for _ in range(args.warmup):
        cpu_sample(threads, seconds_budget=0.0, max_calls=len(LAYER))
    total_bytes = 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        gbs, calls, el = cpu_sample(threads, seconds_budget=0.0, max_calls=len(LAYER))
        per_step.append(time.perf_counter() - t0)
    gbs_steps = [(sum(wbytes(k, n) + (k + n) * 4 for _, k, n in LAYER)) / t / 1e9 for t in per_step]
    value = statistics.median(gbs_steps)
    sample = ("one Llama-2-7B layer's 7 Q4_0 linears at batch 1 per step through the reference route "
              "(forward_linear: full-tensor dequant + f32 row dots, linear.rs:68-87)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * statistics.median(per_step), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[1] Q4_0 Llama-2-7B layer decode (CPU sample: batch 1)",
                   "host_threads": threads},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def gpu_arm(args):
    import numpy as np
    import torch
    import swamp_gpu as sg
    import build_lib

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    if rank == 0:
        build_lib.build()
    if dist:
        dist.barrier()
    gpu = sg.SwampGpu()
    if world > 1:
        uid = gpu.get_unique_id() if rank == 0 else bytes(128)
        t = torch.frombuffer(bytearray(uid), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        gpu.init_rank(rank, world, bytes(t.cpu().numpy().tobytes()), local)
    else:
        gpu.init(1)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # weight generator (host-side synthetic data only)

    n_layers = world  # weak scaling: per-GPU bytes fixed
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    layer_b = sum(wbytes(k, n) for _, k, n in LAYER)
    copies = max(5, int(np.ceil(4.5 * l2 / (layer_b / world))) + 1)
    copies = max(copies, n_layers)
    # register: copies x layer tensors (TP-split when world > 1)
    model = []
    for c in range(copies):
        layer = {}
        for i, (name, k, n) in enumerate(LAYER):
            w = oracle.gen_weight(Q40, SEED, 1000 + 16 * c + i, n, k)
            layer[name] = gpu.register(w, Q40, n, k, TP_MODE[name] if world > 1 else 0)
        model.append(layer)
    # activations / outputs (device, this rank's shard shapes)
    st = torch.cuda.current_stream()
    sp = st.cuda_stream

    def shard(w):
        return w.shard(0)  # n_rows, n_cols, row0, col0

    xs = {b: torch.randn(b, 11008, device="cuda") for b in BATCHES}
    ys = {b: {name: torch.empty(b, 11008, device="cuda") for name, _, _ in LAYER} for b in BATCHES}
    launches_per_call = 2

    def run_layer(layer, b):
        x = xs[b]
        q, kk, v = layer["q"], layer["k"], layer["v"]
        ldx = 11008
        gpu.linear_multi_device([q, kk, v], x.data_ptr(), ldx,
                                [ys[b]["q"].data_ptr(), ys[b]["k"].data_ptr(), ys[b]["v"].data_ptr()],
                                [11008] * 3, b, stream=sp)
        gpu.linear_device(layer["o"], x.data_ptr(), ldx, ys[b]["o"].data_ptr(), 11008, b, stream=sp)
        gpu.linear_multi_device([layer["gate"], layer["up"]], x.data_ptr(), ldx,
                                [ys[b]["gate"].data_ptr(), ys[b]["up"].data_ptr()], [11008] * 2, b, stream=sp)
        gpu.linear_device(layer["down"], x.data_ptr(), ldx, ys[b]["down"].data_ptr(), 11008, b, stream=sp)
        return 4

    state = {"i": 0}

    def step():
        calls = 0
        for b in BATCHES:
            for _ in range(n_layers):
                layer = model[state["i"] % copies]
                state["i"] += 1
                calls += run_layer(layer, b)
        return calls

    # warmup
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    # ------------------------------------------------------------ timed
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(st)
    calls = 0
    for _ in range(args.steps):
        calls += step()
    ev1.record(st)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    total_bytes = step_bytes(n_layers) * args.steps
    value = total_bytes / (ms / 1e3) / 1e9

    # ------------------------------------------ per-launch roofline pass
    # events around each GEMV call of one pass (each call = activation prep +
    # the GEMV kernel, no overlap with its neighbours in this pass)
    per = {}
    for b in BATCHES:
        layer = model[state["i"] % copies]
        state["i"] += 1
        for name, k, n in LAYER:
            if name in ("k", "v", "up"):
                continue
        # time single-tensor calls for the roofline
        for name, k, n in LAYER:
            w = layer[name]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            gpu.linear_device(w, xs[b].data_ptr(), 11008, ys[b][name].data_ptr(), 11008, b, stream=sp)
            e1.record(st)
            per.setdefault(b, []).append((name, k, n, e0, e1))
    torch.cuda.synchronize()
    launch_gbs, launch_us = [], []
    for b, lst in per.items():
        for name, k, n, e0, e1 in lst:
            us = e0.elapsed_time(e1) * 1e3
            by = (wbytes(k, n) + b * (k + n) * 4) / world
            launch_gbs.append(by / (us * 1e-6) / 1e9)
            launch_us.append(us)
    tot_by = sum((wbytes(k, n) + b * (k + n) * 4) / world for b, lst in per.items() for (_, k, n, _, _) in lst)
    tot_us = sum(launch_us)
    achieved = tot_by / (tot_us * 1e-6) / 1e9
    peak, peak_kind = measured_peaks()

    # -------------------------------------------------------------- e2e
    # through the host-pointer C ABI: x copied in and y read back per call
    e2e = None
    if world == 1:
        xh = {b: np.ascontiguousarray(xs[b].cpu().numpy()) for b in BATCHES}
        torch.cuda.synchronize()
        h2d = d2h = 0
        t0 = time.perf_counter()
        e2e_steps = max(1, min(args.steps, 10))
        for _ in range(e2e_steps):
            for b in BATCHES:
                layer = model[state["i"] % copies]
                state["i"] += 1
                x4096 = xh[b][:, :4096]
                outs = gpu.linear_multi([layer["q"], layer["k"], layer["v"]], x4096[0]) if b == 1 else None
                if b == 1:
                    h2d += 4096 * 4
                    d2h += 3 * 4096 * 4
                else:
                    for name in ("q", "k", "v"):
                        gpu.linear(layer[name], x4096)
                        h2d += b * 4096 * 4
                        d2h += b * 4096 * 4
                gpu.linear(layer["o"], x4096)
                h2d += b * 4096 * 4
                d2h += b * 4096 * 4
                for name in ("gate", "up"):
                    gpu.linear(layer[name], x4096)
                    h2d += b * 4096 * 4
                    d2h += b * 11008 * 4
                gpu.linear(layer["down"], xh[b])
                h2d += b * 11008 * 4
                d2h += b * 4096 * 4
        el = time.perf_counter() - t0
        e2e = {"value": round(step_bytes(1) * e2e_steps / el / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d // e2e_steps, "d2h_bytes_per_step": d2h // e2e_steps,
               "path": "sg_linear / sg_linear_multi with host buffers (pinned staging, H2D + D2H per call)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        gbs, ncalls, el = cpu_sample(threads, seconds_budget=args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{ncalls} forward_linear calls (Q4_0 engine route, batch 1) over the layer's 7 "
                         f"tensors in {el:.1f} s on {threads} host threads"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16x2-split/f32-acc (Q4_0 weights)",
            "data": "synthetic (seeded random-init Q4_0 blocks, N(0,1) activations)",
            "config": {"workload": "configs[1]: Llama-2-7B layer Q4_0 linears (4x 4096->4096, 2x 4096->11008, "
                                   "11008->4096) at decode batch 1, 4, 16",
                       "layers_per_step": n_layers, "tp": world, "parallelism": f"tp{world}" if world > 1 else "none",
                       "l2_policy": f"inputs larger than L2: {copies} rotating layer copies "
                                    f"({copies * layer_b / world / 1e6:.0f} MB per GPU vs L2 {l2 / 1e6:.0f} MB)",
                       "bytes_per_step": step_bytes(n_layers)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "gemv_main (decode GEMV) incl. its activation-prep launch",
                         "peak_kind": peak_kind, "per_launch_gbs_median": round(statistics.median(launch_gbs), 1)},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": calls * launches_per_call,
        }
        print(json.dumps(line), flush=True)
    for layer in model:
        for w in layer.values():
            w.free()
    gpu.shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    return gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
